"""Shared parity rules of the GPU tests (not a test module).

Top-k index sets must be identical except at documented near-ties: an index
in the symmetric difference counts as a near-tie when its oracle score lies
within relative ``NEAR_TIE_REL`` of the k-th oracle score (BASELINE
north_star: "top-k index sets identical except at documented near-ties
(relative score gap <1e-3)")."""

from __future__ import annotations

import torch

import oracle as O

NEAR_TIE_REL = 1e-3


def masked_scores(score: torch.Tensor, t_active) -> torch.Tensor:
    """The reference's masked scores (inference.py:5833-5838): score - 1e4 where
    t >= T_active.  score [B, T] fp32; t_active int or [B]."""
    B, T = score.shape
    ta = torch.as_tensor(t_active).reshape(-1).expand(B) if torch.as_tensor(t_active).dim() == 0 \
        else torch.as_tensor(t_active).reshape(-1)
    ramp = torch.arange(T).unsqueeze(0)
    return score.float() - O.TOPK_MASK_AMP * (ramp >= ta.unsqueeze(1)).float()


def assert_topk_sets(got_idx: torch.Tensor, want_idx: torch.Tensor, oracle_masked: torch.Tensor, win: int,
                     what: str = "") -> int:
    """Per row: the valid index sets (values >= 0, offset by ``win``) match
    except for near-ties at the k-th value of the oracle's masked scores.
    Returns the number of near-tie swaps seen."""
    swaps = 0
    for b in range(got_idx.shape[0]):
        g = set(int(v) for v in got_idx[b] if v >= 0)
        w = set(int(v) for v in want_idx[b] if v >= 0)
        assert len(g) == len(w), f"{what} row {b}: {len(g)} valid indices vs {len(w)}"
        if g == w:
            continue
        kth = torch.topk(oracle_masked[b].float(), len(w)).values[-1]
        tol = NEAR_TIE_REL * max(abs(float(kth)), 1e-6)
        for v in g ^ w:
            s = float(oracle_masked[b, v - win])
            assert abs(s - float(kth)) <= tol, \
                f"{what} row {b}: index {v} score {s} vs k-th {float(kth)} is not a near-tie"
        swaps += len(g ^ w) // 2
    return swaps
