"""CPU stand-ins for the reference's Attention / Compressor / Indexer modules
(inference.py:523-623): plain objects carrying the attribute names the
device drop-ins read, filled with seeded random weights, plus the matching
oracle weights and state so one seed drives both sides."""

from __future__ import annotations

from types import SimpleNamespace

import torch

import oracle.path as ref


def _lin(g, out_f, in_f, scale=None):
    s = in_f ** -0.5 if scale is None else scale
    return SimpleNamespace(weight=(torch.randn(out_f, in_f, generator=g) * s).to(torch.bfloat16))


def _norm(g, d, eps=1e-6):
    return SimpleNamespace(weight=1.0 + 0.02 * torch.randn(d, generator=g), eps=eps)


def make_block(seed: int = 0, B: int = 2, dim: int = 256, q_lora: int = 128, o_lora: int = 64,
               max_seq_len: int = 1024, index_topk: int = 512, H: int = 64, D: int = 512, Hi: int = 64,
               Di: int = 128, rd: int = 64, W: int = 128, r: int = 4, G: int = 8):
    """Returns (attn stand-in, oracle BlockWeights, oracle LayerState)."""
    g = torch.Generator().manual_seed(seed)
    cos, sin = ref.rope_tables(rd, max_seq_len, compressed=True)
    freqs = torch.complex(cos, sin)
    T = max_seq_len // r

    def compressor(d, rotate):
        kv_state, score_state = ref.compressor_init_state(B, d, r, True)
        return SimpleNamespace(head_dim=d, rope_head_dim=rd, compress_ratio=r, overlap=True, rotate=rotate,
                               ape=0.1 * torch.randn(r, 2 * d, generator=g), wkv=_lin(g, 2 * d, dim),
                               wgate=_lin(g, 2 * d, dim), norm=_norm(g, d), kv_state=kv_state,
                               score_state=score_state, kv_cache=None, freqs_cis=freqs)

    comp = compressor(D, False)
    icomp = compressor(Di, True)
    indexer = SimpleNamespace(head_dim=Di, rope_head_dim=rd, n_heads=Hi, n_local_heads=Hi, compress_ratio=r,
                              softmax_scale=Di ** -0.5, index_topk=index_topk, freqs_cis=freqs,
                              wq_b=_lin(g, Hi * Di, q_lora), weights_proj=_lin(g, Hi, dim), compressor=icomp,
                              kv_cache=torch.zeros(B, T, Di))
    attn = SimpleNamespace(
        dim=dim, n_heads=H, n_local_heads=H, head_dim=D, rope_head_dim=rd, q_lora_rank=q_lora,
        n_groups=G, n_local_groups=G, o_lora_rank=o_lora, softmax_scale=D ** -0.5, eps=1e-6, window_size=W,
        compress_ratio=r, freqs_cis=freqs, attn_sink=torch.randn(H, generator=g),
        q_norm=_norm(g, q_lora), kv_norm=_norm(g, D), wq_a=_lin(g, q_lora, dim), wq_b=_lin(g, H * D, q_lora),
        wkv=_lin(g, D, dim), wo_a=_lin(g, G * o_lora, H * D // G), wo_b=_lin(g, dim, G * o_lora),
        kv_cache=torch.zeros(B, W + T, D), compressor=comp, indexer=indexer)
    bw = ref.BlockWeights(
        wq_a=attn.wq_a.weight, q_norm=attn.q_norm.weight, wq_b=attn.wq_b.weight, wkv=attn.wkv.weight,
        kv_norm=attn.kv_norm.weight, wo_a=attn.wo_a.weight, wo_b=attn.wo_b.weight, c_wkv=comp.wkv.weight,
        c_wgate=comp.wgate.weight, i_wq_b=indexer.wq_b.weight, i_wproj=indexer.weights_proj.weight,
        i_wkv=icomp.wkv.weight, i_wgate=icomp.wgate.weight, n_groups=G)
    st = ref.LayerState(
        kv_cache=torch.zeros(B, W + T, D, dtype=torch.bfloat16),
        idx_kv_cache=torch.zeros(B, T, Di, dtype=torch.bfloat16),
        cmp_kv=comp.kv_state.clone(), cmp_sc=comp.score_state.clone(),
        icmp_kv=icomp.kv_state.clone(), icmp_sc=icomp.score_state.clone(),
        ape=comp.ape, gamma=comp.norm.weight, iape=icomp.ape, igamma=icomp.norm.weight,
        sink=attn.attn_sink, cos=cos, sin=sin, win=W, ratio=r, index_topk=index_topk, scale=1.0)
    return attn, bw, st
