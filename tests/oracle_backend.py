"""The CPU oracle behind the ``dsv4attn.ops`` call signatures, so host-side
orchestration (the sequence split's shard offsets, exchanges and window
ownership) can run in gloo processes on CPU with the oracle as the checker.
Test infrastructure only; the shipped package never imports it."""

from __future__ import annotations

import torch

import oracle.path as ref


def _pos_list(pos):
    return [int(p) for p in pos.reshape(-1).tolist()]


class OracleOps:
    """Same names, arguments and in-place outputs as dsv4attn.ops."""

    @staticmethod
    def kv_window_write(kv, kv_cache, pos, win, rope_dim=64, scales=None):
        row, _, _ = ref.kv_quant_row(kv, rope_dim)
        for b, p in enumerate(_pos_list(pos)):
            kv_cache[b, p % win] = row[b]

    @staticmethod
    def compressor_step(kv_row, score_row, ape, kv_state, score_state, gamma, cos, sin, kv_cache, slot_offset, pos,
                        ratio, overlap, rotate=False, eps=1e-6, rope_dim=64, emitted=None, write_state=True):
        rows = kv_cache.shape[1]
        for b, p in enumerate(_pos_list(pos)):
            ks, ss = kv_state[b:b + 1], score_state[b:b + 1]
            ref.compressor_state_write(ks, ss, kv_row[b:b + 1], score_row[b:b + 1], ape, p, ratio, overlap)
            if (p + 1) % ratio:
                continue
            out_row = slot_offset + p // ratio
            if 0 <= out_row < rows:
                c = p + 1 - ratio
                kv_cache[b, out_row] = ref.compressor_emit(ks, ss, gamma, cos[c], sin[c], ratio, overlap, rope_dim,
                                                           eps, rotate)[0]
            if overlap:
                ks.copy_(ref.shift_matrix_apply(ks, ratio))
                ss.copy_(ref.shift_matrix_apply(ss, ratio))

    @staticmethod
    def shard_active(t_active, lo, n_local, out=None):
        out.copy_((t_active - lo).clamp(0, n_local))
        return out

    @staticmethod
    def indexer_score(q, k_cache, w, T, out=None, t_valid=None):
        out[:, :T] = ref.indexer_score(q, k_cache[:, :T], w)
        return out

    @staticmethod
    def indexer_topk(score, t_active, k, win, T=None, sort_desc=False, mask_mode=0, out=None, out_score=None,
                     ws=None):
        T = score.shape[1] if T is None else T
        ta = t_active.reshape(-1)
        masked = score[:, :T].float() - ref.TOPK_MASK_AMP * (torch.arange(T).unsqueeze(0) >= ta.unsqueeze(1)).float()
        if mask_mode == 1:
            masked = masked.masked_fill(torch.arange(T).unsqueeze(0) >= ta.unsqueeze(1), float("-inf"))
        for b in range(score.shape[0]):
            order = sorted(range(T), key=lambda t: (-float(masked[b, t]), t))[:k]
            if not sort_desc:
                order = sorted(order)
            vals = masked[b, order]
            out[b] = torch.where(vals >= ref.TOPK_VALID_MIN, torch.tensor(order, dtype=torch.int32) + win,
                                 torch.full((k,), -1, dtype=torch.int32))
            if out_score is not None:
                out_score[b] = vals
        return out

    @staticmethod
    def topk_merge(cand_score, cand_idx, k, win, out=None, out_score=None):
        for b in range(cand_score.shape[0]):
            s, i = ref.topk_merge(cand_score[b], cand_idx[b], k)
            out[b] = torch.where((s >= ref.TOPK_VALID_MIN) & (i >= 0), i + win, torch.full_like(i, -1))
            if out_score is not None:
                out_score[b] = s
        return out

    @staticmethod
    def window_indices(pos, win, out=None):
        for b, p in enumerate(_pos_list(pos)):
            out[b] = ref.window_indices(p, win)
        return out

    @staticmethod
    def shard_local_indices(sel, lo, hi, W, win_idx=None, local_base=0, win_base=0, out=None):
        if win_idx is None:
            out[:, :W] = -1
        else:
            out[:, :W] = torch.where(win_idx >= 0, win_idx + win_base, torch.full_like(win_idx, -1))
        out[:, W:] = torch.where((sel >= lo) & (sel < hi), sel - lo + local_base, torch.full_like(sel, -1))
        return out

    @staticmethod
    def sparse_attn_partial(q, kv, idx, scale, part_ml=None, part_o=None, ws=None, status=None):
        m, l, o = ref.sparse_attn_partial(q, kv, idx, scale)
        part_ml[..., 0] = m
        part_ml[..., 1] = l
        part_o.copy_(o)
        return part_ml, part_o

    @staticmethod
    def lse_combine(part_ml, part_o, sink, out=None):
        parts = [(part_ml[g, ..., 0], part_ml[g, ..., 1], part_o[g]) for g in range(part_ml.shape[0])]
        out.copy_(ref.lse_combine(parts, sink.unsqueeze(0)).to(out.dtype))
        return out

    @staticmethod
    def lse_combine_strided(part_ml, ml_pstride, part_o, o_pstride, P, M, H, D, sink, out):
        ml = torch.stack([part_ml[p * ml_pstride:p * ml_pstride + M * H * 2].view(M, H, 2) for p in range(P)])
        o = torch.stack([part_o[p * o_pstride:p * o_pstride + M * H * D].view(M, H, D) for p in range(P)])
        return OracleOps.lse_combine(ml, o, sink, out=out)

    @staticmethod
    def advance_positions(pos, t_active, ratio, step=1):
        pos += step
        if t_active is not None:
            t_active.copy_((pos + 1) // ratio)
