"""The path across GPUs: batch split and sequence split.

Batch split (config 2): the sequences are independent, so each rank owns
B / world of them with their caches and runs ``layer.DecodePath`` unchanged;
there is no collective on the data path (``batch_shard``).

Sequence split (config 3): one long context, its compressed KV rows and
indexer keys cut into ``world`` contiguous shards [lo, hi).  One decode step
of one layer on every rank:

  local    window ring write (replicated; attended by the last rank, which
           holds the newest tokens), both compressors (state replicated,
           the emitted row stored only by the rank that owns its position),
           indexer score over the shard, local top-k' candidates
           (k' = min(k, shard rows)) with global positions
  exchange one all-gather of the candidates (G x k' x 8 bytes)
  attend   global merge (identical on every rank), this shard's rows of the
           selection, partial attention (m, l, o) without the sink
  exchange one all-gather of the partials (G x H x (D + 2) x 4 bytes)
  combine  log-sum-exp merge with the sink counted once -> bf16 o

Any global top-k entry is in its shard's top-k', and both selections break
ties towards the lower position, so the merged index set is exactly the
unsplit one (inference.py:5823-5851); the combine is exact up to fp32
rounding.  The reference plans this split (briefs/future_max_utilization.md:
177-204) but does not implement it.

``SeqShard`` holds one rank's buffers and runs the three compute phases;
``SeqSplitPath`` drives it with a comm: ``P2PComm`` (peer-memory stores
over NVLink with per-rank flags, the GPU default) or ``TorchDistComm``
(all-gathers over a process group: NCCL, or gloo in the CPU tests).  The phases are separate methods so that G shards can also be
driven inside one process (the exchanges become copies), which is how the
single-GPU tests check the split against the unsplit path.
"""

from __future__ import annotations

import torch

from . import ops as native_ops
from .layer import LayerInputs
from .tables import PathArgs, rope_cos_sin

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def batch_shard(B_total: int, rank: int, world: int):
    """Contiguous [start, stop) of the sequences rank ``rank`` owns."""
    if B_total % world:
        raise ValueError(f"batch {B_total} not divisible by {world} ranks")
    per = B_total // world
    return rank * per, (rank + 1) * per


def seq_shard(T_total: int, rank: int, world: int):
    """Contiguous [lo, hi) of the compressed positions rank ``rank`` owns."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    per = -(-T_total // world)
    lo = min(rank * per, T_total)
    return lo, min(lo + per, T_total)


class TorchDistComm:
    """The two exchanges as all-gathers over a torch.distributed process
    group (NCCL on GPUs, gloo in the CPU tests)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        """out [world, *inp.shape] <- every rank's inp."""
        try:
            self.dist.all_gather_into_tensor(out, inp, group=self.group)
        except (RuntimeError, NotImplementedError):
            self.dist.all_gather(list(out.unbind(0)), inp, group=self.group)

    def exchange(self, L, phase: int) -> None:
        if phase == 0:
            self.all_gather(L.cand_all, L.cand)
        else:
            self.all_gather(L.part_all, L.part)

    def end_step(self) -> None:
        pass

    def close(self) -> None:
        pass


class P2PComm:
    """The two exchanges as peer-memory stores over NVLink (dsa_p2p_*):
    every rank publishes its candidates / partials straight into slot
    ``rank`` of every peer's receive buffer and raises its flag there; the
    consumer waits (bounded) on the G flags of that layer and phase.  The
    receive buffers of all layers live in one arena per rank, exported once
    as a CUDA IPC handle and mapped by the other ranks of the node.  Set-up
    uses the process group once (an object all-gather of the handles)."""

    def __init__(self, shard: "SeqShard", group=None):
        import ctypes
        import torch.distributed as dist
        if shard.arena is None:
            raise ValueError("P2PComm needs a SeqShard built with peer_exchange=True")
        L = native_ops.lib()
        self.shard = shard
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world != shard.world or self.rank != shard.rank:
            raise ValueError("process group and shard disagree on rank / world")
        dev = shard.device
        base = shard.arena.buf.data_ptr()
        hsize = int(L.dsa_p2p_handle_size())
        h = ctypes.create_string_buffer(hsize)
        off = ctypes.c_uint64(0)
        native_ops.check(L.dsa_p2p_export(ctypes.c_void_p(base), h, ctypes.byref(off)), "p2p_export")
        mine = (bytes(h.raw), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self.mapped = []
        peer_base = []
        for g, (hb, o) in enumerate(allh):
            if g == self.rank:
                peer_base.append(base)
                continue
            p = ctypes.c_void_p(0)
            native_ops.check(L.dsa_p2p_import(ctypes.create_string_buffer(hb, hsize), ctypes.byref(p)),
                             "p2p_import")
            self.mapped.append(p.value)
            peer_base.append(p.value + o)
        self.epoch = torch.ones(1, dtype=I32, device=dev)
        # per layer and phase: device arrays of the G destination and flag addresses
        self.routes = []
        for Ly in shard.layers:
            per = []
            for phase, recv in ((0, Ly.cand_all), (1, Ly.part_all)):
                slot = recv[self.rank].data_ptr() - base
                flag = Ly.flags[phase, self.rank].data_ptr() - base
                dst = torch.tensor([pb + slot for pb in peer_base], dtype=torch.int64, device=dev)
                fl = torch.tensor([pb + flag for pb in peer_base], dtype=torch.int64, device=dev)
                per.append((dst, fl))
            self.routes.append(per)
        self.layer_index = {id(Ly): i for i, Ly in enumerate(shard.layers)}
        dist.barrier(group=group)

    def exchange(self, L, phase: int) -> None:
        lib = native_ops.lib()
        src = L.cand if phase == 0 else L.part
        dst, fl = self.routes[self.layer_index[id(L)]][phase]
        st = torch.cuda.current_stream(src.device).cuda_stream
        native_ops.check(lib.dsa_p2p_publish(src.data_ptr(), src.numel() * src.element_size(), dst.data_ptr(),
                                             fl.data_ptr(), self.epoch.data_ptr(), self.world,
                                             L.done[phase].data_ptr(), st), "p2p_publish")
        native_ops.check(lib.dsa_p2p_wait(L.flags[phase].data_ptr(), self.world, self.epoch.data_ptr(),
                                          self.shard.status.data_ptr(), st), "p2p_wait")

    def end_step(self) -> None:
        native_ops.check(native_ops.lib().dsa_counter_bump(self.epoch.data_ptr(),
                                                           torch.cuda.current_stream(self.epoch.device).cuda_stream),
                         "counter_bump")

    def close(self) -> None:
        lib = native_ops.lib()
        for p in self.mapped:
            lib.dsa_p2p_close(p)
        self.mapped = []


class _Arena:
    """Bump allocator over one zeroed device buffer: the receive buffers
    peers write into must share one allocation (one IPC export)."""

    def __init__(self, nbytes: int, device):
        self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        self.off = 0

    def take(self, shape, dtype) -> torch.Tensor:
        n = 1
        for x in shape:
            n *= x
        nb = n * torch.tensor([], dtype=dtype).element_size()
        if self.off + nb > self.buf.numel():
            raise RuntimeError("exchange arena too small")
        t = self.buf[self.off:self.off + nb].view(dtype).view(shape)
        self.off += -(-nb // 256) * 256
        return t

    @staticmethod
    def layer_bytes(B: int, kc: int, world: int, H: int, D: int) -> int:
        r = lambda nb: -(-nb // 256) * 256
        return r(world * 2 * B * kc * 4) + r(world * B * H * (D + 2) * 4) + r(2 * world * 4) + r(2 * world * 4)


class SeqShardLayer:
    """One layer's shard: compressed rows [lo, hi) + the window ring."""

    def __init__(self, args: PathArgs, B: int, n_local: int, k: int, kc: int, world: int, device,
                 arena: _Arena | None = None):
        D, Di, H, W, r = args.head_dim, args.index_head_dim, args.n_heads, args.window_size, args.compress_ratio
        dev = device
        # rows [0, n_local) compressed entries of this shard, then the W-row window ring
        self.kv = torch.zeros(B, n_local + W, D, dtype=BF16, device=dev)
        self.keys = torch.zeros(B, max(n_local, 1), Di, dtype=BF16, device=dev)
        self.cmp_kv = torch.zeros(B, 2 * r, 2 * D, dtype=F32, device=dev)
        self.cmp_sc = torch.full((B, 2 * r, 2 * D), float("-inf"), dtype=F32, device=dev)
        self.icmp_kv = torch.zeros(B, 2 * r, 2 * Di, dtype=F32, device=dev)
        self.icmp_sc = torch.full((B, 2 * r, 2 * Di), float("-inf"), dtype=F32, device=dev)
        self.ape = torch.zeros(r, 2 * D, dtype=F32, device=dev)
        self.gamma = torch.ones(D, dtype=F32, device=dev)
        self.iape = torch.zeros(r, 2 * Di, dtype=F32, device=dev)
        self.igamma = torch.ones(Di, dtype=F32, device=dev)
        self.sink = torch.zeros(H, dtype=F32, device=dev)
        # per-step scratch
        self.score = torch.zeros(B, max(n_local, 1), dtype=F32, device=dev)
        # candidates, one flat buffer so one all-gather moves them: B*kc fp32
        # scores, then B*kc int32 global positions
        self.kc = kc
        self.cand = torch.empty(2 * B * kc, dtype=I32, device=dev)
        self.cand_score = self.cand[:B * kc].view(F32).view(B, kc)
        self.cand_idx = self.cand[B * kc:].view(B, kc)
        self.cand_score.fill_(float("-inf"))
        self.cand_idx.fill_(-1)
        take = arena.take if arena is not None else (lambda shape, dt: torch.zeros(shape, dtype=dt, device=dev))
        self.cand_all = take((world, 2 * B * kc), I32)
        self.sel = torch.full((B, k), -1, dtype=I32, device=dev)
        self.selected = self.sel     # the merged selection of the last step (a view of sel or cand_idx)
        self.lidx = torch.full((B, W + k), -1, dtype=I32, device=dev)
        # the partial (m, l) and o in one flat buffer as well: B*H*2, then B*H*D floats
        self.part = torch.zeros(B * H * (D + 2), dtype=F32, device=dev)
        self.pml = self.part[:B * H * 2].view(B, H, 2)
        self.po = self.part[B * H * 2:].view(B, H, D)
        self.part_all = take((world, B * H * (D + 2)), F32)
        # peer-exchange bookkeeping: per phase (0 candidates, 1 partials) one
        # flag per source rank, and the publish kernel's per-destination counters
        self.flags = take((2, world), I32)
        self.done = take((2, world), I32)

    def cand_all_views(self, B: int):
        """(scores [G, B, kc], positions [G, B, kc]) views of the gathered candidates."""
        G = self.cand_all.shape[0]
        n = B * self.kc
        return (self.cand_all[:, :n].view(F32).view(G, B, self.kc), self.cand_all[:, n:].view(G, B, self.kc))

    def part_all_views(self, B: int, H: int, D: int):
        G = self.part_all.shape[0]
        return (self.part_all[:, :B * H * 2].view(G, B, H, 2), self.part_all[:, B * H * 2:].view(G, B, H, D))

    def kv_compressed(self, n_local: int):
        return self.kv[:, :n_local]

    def kv_window(self, n_local: int):
        return self.kv[:, n_local:]


class SeqShard:
    """One rank's part of the sequence split for a stack of layers."""

    def __init__(self, args: PathArgs, B: int, T_total: int, rank: int, world: int, device, k: int | None = None,
                 n_layers: int = 1, max_seq_len: int | None = None, window_rank: int | None = None,
                 scale: float | None = None, backend=None, peer_exchange: bool = False):
        self.args = args
        self.B = B
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.ops = backend if backend is not None else native_ops
        self.T_total = T_total
        self.lo, self.hi = seq_shard(T_total, rank, world)
        self.n_local = self.hi - self.lo
        self.k = args.index_topk if k is None else k
        if self.k > T_total:
            raise ValueError(f"index_topk {self.k} > compressed capacity {T_total}")
        per = -(-T_total // world)
        self.kc = min(self.k, per)
        if world * self.kc > 16384:
            raise ValueError(f"{world} x {self.kc} candidates exceed the 16384 the merge selects from")
        self.window_rank = world - 1 if window_rank is None else window_rank
        self.scale = args.softmax_scale if scale is None else scale
        max_seq = max_seq_len if max_seq_len is not None else T_total * args.compress_ratio
        self.cos, self.sin = rope_cos_sin(args, max_seq, compressed=True, device=self.device)
        self.arena = None
        if peer_exchange:
            self.arena = _Arena(n_layers * _Arena.layer_bytes(B, self.kc, world, args.n_heads, args.head_dim),
                                self.device)
        self.layers = [SeqShardLayer(args, B, self.n_local, self.k, self.kc, world, self.device, self.arena)
                       for _ in range(n_layers)]
        dev = self.device
        self.pos = torch.zeros(B, dtype=I32, device=dev)
        self.t_active = torch.zeros(B, dtype=I32, device=dev)
        self.t_local = torch.zeros(B, dtype=I32, device=dev)
        self.status = torch.zeros(1, dtype=I32, device=dev)
        self.win_idx = torch.full((B, args.window_size), -1, dtype=I32, device=dev)
        self.side = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        H, D = args.n_heads, args.head_dim
        ws_attn = 0
        # few long rows: the multi-CTA top-k (one CTA per row would idle the GPU)
        self.use_wide = backend is None and B <= 4
        self.wide_ws = None
        if backend is None:
            ws_attn = int(native_ops.lib().dsa_sparse_attn_workspace_size(B, 1, H, D, args.window_size + self.k))
            ws_topk = int(native_ops.lib().dsa_indexer_topk_workspace_size(B, max(self.n_local, 1), self.kc))
            self.ws = native_ops.Workspace(dev, max(ws_attn, ws_topk))
            if self.use_wide:
                self.wide_ws = native_ops.WideTopkWorkspace(dev)
                self.wide_ws.get(B, max(self.n_local, 1))
                self.wide_ws.get(B, world * self.kc)
        else:
            self.ws = None

    def set_positions(self, pos) -> None:
        p = torch.as_tensor(pos, dtype=I32).reshape(-1).expand(self.B).contiguous()
        self.pos.copy_(p.to(self.device))
        self.t_active.copy_(((p + 1) // self.args.compress_ratio).to(self.device))
        self._per_step()

    def _per_step(self) -> None:
        """What depends only on the positions, once per step for all layers:
        this shard's T_active and the window ring indices."""
        o, n = self.ops, self.n_local
        o.shard_active(self.t_active, self.lo, n, out=self.t_local)
        if self.rank == self.window_rank:
            o.window_indices(self.pos, self.args.window_size, out=self.win_idx)

    # ---- phase 1: everything before the candidate exchange
    def phase_local(self, L: SeqShardLayer, x: LayerInputs) -> None:
        a, o = self.args, self.ops
        W, r, n = a.window_size, a.compress_ratio, self.n_local
        side = self.side
        if side is not None:
            # window write and attention compressor feed only the attention:
            # a side branch, joined in phase_attend
            side.wait_stream(torch.cuda.current_stream(self.device))
            ctx = torch.cuda.stream(side)
        else:
            ctx = _nullctx()
        with ctx:
            o.kv_window_write(x.kv, L.kv_window(n), self.pos, W, rope_dim=a.rope_head_dim)
            o.compressor_step(x.cmp_kv, x.cmp_score, L.ape, L.cmp_kv, L.cmp_sc, L.gamma, self.cos, self.sin,
                              L.kv_compressed(max(n, 1)) if n else L.kv[:, :1], -self.lo if n else -(1 << 30),
                              self.pos, r, overlap=True, rotate=False, eps=a.norm_eps, rope_dim=a.rope_head_dim)
        o.compressor_step(x.icmp_kv, x.icmp_score, L.iape, L.icmp_kv, L.icmp_sc, L.igamma, self.cos, self.sin,
                          L.keys[:, :max(n, 1)], -self.lo, self.pos, r, overlap=True, rotate=False, eps=a.norm_eps,
                          rope_dim=a.rope_head_dim)
        if n == 0:
            return
        o.indexer_score(x.iq, L.keys, x.iw, n, out=L.score, t_valid=self.t_local)
        kn = min(self.kc, n)
        if self.use_wide:
            o.topk_wide(L.score, kn, self.lo, t_active=self.t_local, T=n, mask_mode=1, out=L.cand_idx[:, :kn],
                        out_score=L.cand_score[:, :kn], ws=self.wide_ws, status=self.status)
        else:
            o.indexer_topk(L.score, self.t_local, kn, self.lo, T=n, sort_desc=False, mask_mode=1,
                           out=L.cand_idx[:, :kn], out_score=L.cand_score[:, :kn], ws=self.ws)

    # ---- phase 2: merge, local rows of the selection, partial attention
    def phase_attend(self, L: SeqShardLayer, x: LayerInputs, out: torch.Tensor | None = None) -> None:
        """With ``out`` and a single shard the attention writes the final
        output (sink included) and no partial exchange or combine follows."""
        a, o = self.args, self.ops
        W, r, n = a.window_size, a.compress_ratio, self.n_local
        G, B, kc = self.world, self.B, self.kc
        if G == 1 and kc == self.k:
            L.selected = L.cand_idx          # one shard: its candidates are the global top-k
        else:
            if self.use_wide:
                # row b of rank g's list sits at g * 2*B*kc + b*kc: read the
                # gathered buffer in place as G segments per row; the lists
                # arrive in ascending position order, rank by rank, so the
                # lower-slot tie rule is the lower-position rule
                flat = L.cand_all.view(-1)
                o.topk_wide(flat.view(F32), self.k, 0,
                            ids=flat[B * kc:], mask_mode=0, out=L.sel, ws=self.wide_ws, status=self.status,
                            seg_len=kc, seg_stride=2 * B * kc, B=B, T=G * kc, ld_score=kc)
            else:
                sc, ix = L.cand_all_views(B)
                cs = sc.permute(1, 0, 2).reshape(B, G * kc)
                ci = ix.permute(1, 0, 2).reshape(B, G * kc)
                o.topk_merge(cs, ci, self.k, 0, out=L.sel)
            L.selected = L.sel
        attend_window = self.rank == self.window_rank
        o.shard_local_indices(L.selected, self.lo, self.hi, W, self.win_idx if attend_window else None,
                              local_base=0, win_base=n, out=L.lidx)
        if self.side is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.side)
        if out is not None:
            if G != 1:
                raise ValueError("a final output from phase_attend needs a single shard")
            o.sparse_attn(x.q, L.kv, L.lidx, L.sink, self.scale, out=out.view(B, a.n_heads, a.head_dim), ws=self.ws,
                          status=self.status)
            return
        o.sparse_attn_partial(x.q, L.kv, L.lidx, self.scale, part_ml=L.pml, part_o=L.po, ws=self.ws,
                              status=self.status)

    # ---- phase 3: combine the gathered partials
    def phase_combine(self, L: SeqShardLayer, out: torch.Tensor) -> None:
        B, H, D = self.B, self.args.n_heads, self.args.head_dim
        ps = B * H * (D + 2)
        flat = L.part_all.view(-1)
        self.ops.lse_combine_strided(flat, ps, flat[B * H * 2:], ps, self.world, B, H, D, L.sink,
                                     out.view(B, H, D))

    def advance(self) -> None:
        self.ops.advance_positions(self.pos, self.t_active, self.args.compress_ratio, 1)
        self._per_step()


class SeqSplitPath:
    """Runs a SeqShard's layers with the two exchanges between phases (a
    single shard needs no comm: ``comm=None``)."""

    def __init__(self, shard: SeqShard, comm=None):
        if comm is None and shard.world != 1:
            raise ValueError("a split over several ranks needs a comm")
        self.shard = shard
        self.comm = comm

    def layer_step(self, L: SeqShardLayer, x: LayerInputs, out: torch.Tensor) -> None:
        s, c = self.shard, self.comm
        if s.world == 1:
            # one shard: its candidates are the selection and its attention the result
            s.phase_local(L, x)
            s.phase_attend(L, x, out)
            return
        s.phase_local(L, x)
        c.exchange(L, 0)
        s.phase_attend(L, x)
        c.exchange(L, 1)
        s.phase_combine(L, out)

    def step(self, inputs, outs, advance: bool = True) -> None:
        for L, x, o in zip(self.shard.layers, inputs, outs):
            self.layer_step(L, x, o)
        if self.comm is not None:
            self.comm.end_step()
        if advance:
            self.shard.advance()


def run_shards_in_process(shards, inputs, outs, advance: bool = True) -> None:
    """One step of all G shards of a sequence split inside one process (the
    exchanges become copies).  ``inputs[l]`` is shared by every shard (the
    replicated per-token inputs); ``outs[g][l]`` receives shard g's result."""
    G = len(shards)
    for li in range(len(shards[0].layers)):
        Ls = [s.layers[li] for s in shards]
        for s, L in zip(shards, Ls):
            s.phase_local(L, inputs[li])
        for L in Ls:
            for g in range(G):
                L.cand_all[g].copy_(Ls[g].cand)
        for s, L in zip(shards, Ls):
            s.phase_attend(L, inputs[li])
        for L in Ls:
            for g in range(G):
                L.part_all[g].copy_(Ls[g].part)
        for g, (s, L) in enumerate(zip(shards, Ls)):
            s.phase_combine(L, outs[g][li])
    if advance:
        for s in shards:
            s.advance()
