"""A seeded sequence-split case shared by the CPU (gloo) and GPU tests: the
full context state, its per-shard slices, the per-step inputs and the
unsplit oracle state."""

from __future__ import annotations

from types import SimpleNamespace

import torch

import oracle.path as ref
from dsv4attn.layer import LayerInputs
from dsv4attn.tables import PathArgs

BF16 = torch.bfloat16


def make_case(seed: int, B: int, T_total: int, W: int, k: int, steps: int, pos0: int):
    args = PathArgs(window_size=W, index_topk=k)
    D, Di, H, Hi, r = args.head_dim, args.index_head_dim, args.n_heads, args.index_n_heads, args.compress_ratio
    g = torch.Generator().manual_seed(seed)
    t0 = (pos0 + 1) // r

    def rn(*shape, s=1.0):
        return torch.randn(*shape, generator=g) * s

    comp = rn(B, T_total, D).to(BF16)
    comp[:, t0:] = 0
    keys = rn(B, T_total, Di).to(BF16)
    keys[:, t0:] = 0
    full = SimpleNamespace(
        comp=comp, keys=keys, win=rn(B, W, D).to(BF16),
        cmp_kv=rn(B, 2 * r, 2 * D).to(BF16).float(), cmp_sc=rn(B, 2 * r, 2 * D).to(BF16).float(),
        icmp_kv=rn(B, 2 * r, 2 * Di).to(BF16).float(), icmp_sc=rn(B, 2 * r, 2 * Di).to(BF16).float(),
        ape=rn(r, 2 * D, s=0.1), gamma=1 + rn(D, s=0.02), iape=rn(r, 2 * Di, s=0.1), igamma=1 + rn(Di, s=0.02),
        sink=rn(H))
    inputs = []
    for _ in range(steps):
        inputs.append(LayerInputs(
            q=rn(B, H, D).to(BF16), kv=rn(B, D).to(BF16), cmp_kv=rn(B, 2 * D).to(BF16),
            cmp_score=rn(B, 2 * D).to(BF16), iq=rn(B, Hi, Di).to(BF16), icmp_kv=rn(B, 2 * Di).to(BF16),
            icmp_score=rn(B, 2 * Di).to(BF16), iw=rn(B, Hi, s=0.02)))
    return args, full, inputs


def load_shard(shard, full) -> None:
    """Copy the shard's slice of the full state into its first layer."""
    L = shard.layers[0]
    lo, hi, n = shard.lo, shard.hi, shard.n_local
    dev = L.kv.device
    L.kv[:, :n] = full.comp[:, lo:hi].to(dev)
    L.kv[:, n:] = full.win.to(dev)
    L.keys[:, :n] = full.keys[:, lo:hi].to(dev)
    for name in ("cmp_kv", "cmp_sc", "icmp_kv", "icmp_sc", "ape", "gamma", "iape", "igamma", "sink"):
        getattr(L, name).copy_(getattr(full, name).to(dev))


def oracle_state(args, full, max_seq_len: int):
    cos, sin = ref.rope_tables(args.rope_head_dim, max_seq_len, compressed=True)
    return ref.LayerState(
        kv_cache=torch.cat([full.win, full.comp], dim=1).clone(), idx_kv_cache=full.keys.clone(),
        cmp_kv=full.cmp_kv.clone(), cmp_sc=full.cmp_sc.clone(), icmp_kv=full.icmp_kv.clone(),
        icmp_sc=full.icmp_sc.clone(), ape=full.ape, gamma=full.gamma, iape=full.iape, igamma=full.igamma,
        sink=full.sink, cos=cos, sin=sin, win=args.window_size, ratio=args.compress_ratio,
        index_topk=args.index_topk, scale=args.softmax_scale)


def oracle_outputs(args, full, inputs, pos0: int, max_seq_len: int, with_scores: bool = False):
    """The unsplit oracle's outputs and index rows per step (and, with
    ``with_scores``, its indexer scores [B, T_active] per step)."""
    st = oracle_state(args, full, max_seq_len)
    outs, idxs, scores = [], [], []
    for s, x in enumerate(inputs):
        o, idx = ref.decode_layer_step(st, pos0 + s, x.q, x.kv, x.cmp_kv, x.cmp_score, x.iq, x.icmp_kv,
                                       x.icmp_score, x.iw)
        outs.append(o)
        idxs.append(idx)
        scores.append(st.extra["score"])
    if with_scores:
        return outs, idxs, scores
    return outs, idxs
