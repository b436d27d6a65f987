"""GPU parity of the sequence split (config 3), all shards driven in one
process on one GPU (the exchanges become copies; the multi-rank NCCL run
is bench.py --workload cfg3 under torchrun).

* small contexts: every shard's combined output equals the unsplit oracle
  step (rtol/atol 2e-2) and the merged selection equals the oracle's top-k
  set except at near-ties;
* the config-3 size (65536 compressed entries, top-2048): the 1-, 2- and
  8-way splits each select the oracle's top-k set except at near-ties and
  match its output; the G-way selection also equals the 1-way one exactly
  (the split is exact by construction)."""

import pytest
import torch

from parity import assert_topk_sets, masked_scores
from seqsplit_case import load_shard, make_case, oracle_outputs

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


def _run_split(args, full, inputs, G, T_total, pos0, max_seq, dev, B):
    from dsv4attn.dist import SeqShard, run_shards_in_process
    shards = [SeqShard(args, B, T_total, g, G, dev, k=args.index_topk, max_seq_len=max_seq) for g in range(G)]
    for s in shards:
        load_shard(s, full)
        s.set_positions(pos0)
    outs_all, sels = [], []
    for x in inputs:
        xd = type(x)(*[t.to(dev) for t in x.tensors()])
        outs = [[torch.empty(B, args.n_heads, args.head_dim, dtype=BF16, device=dev)] for _ in range(G)]
        run_shards_in_process(shards, [xd], outs)
        torch.cuda.synchronize()
        outs_all.append([o[0].cpu() for o in outs])
        sels.append(shards[0].layers[0].selected.cpu().clone())
        for s in shards:
            assert int(s.status.item()) == 0
    return outs_all, sels


@pytest.mark.parametrize("G,B", [(1, 1), (2, 1), (3, 2), (8, 1)])
def test_seq_split_matches_unsplit_oracle(cuda_dev, G, B):
    T_total, W, k, steps = 4096, 128, 512, 6
    pos0 = 4 * T_total - 1 - steps - 3
    max_seq = 4 * T_total + 64
    args, full, inputs = make_case(100 + G, B, T_total, W, k, steps, pos0)
    want, want_idx, want_score = oracle_outputs(args, full, inputs, pos0, max_seq, with_scores=True)
    outs, sels = _run_split(args, full, inputs, G, T_total, pos0, max_seq, cuda_dev, B)
    for s in range(steps):
        for g in range(G):
            assert torch.allclose(outs[s][g].float(), want[s].float(), rtol=2e-2, atol=2e-2), (s, g)
        t_active = (pos0 + s + 1) // 4
        got = torch.where(sels[s] >= 0, sels[s] + W, torch.full_like(sels[s], -1))
        assert_topk_sets(got, want_idx[s][:, W:], masked_scores(want_score[s], t_active), W, what=f"step {s}")


def test_seq_split_config3_size_matches_oracle(cuda_dev):
    T_total, W, k, steps = 65536, 128, 2048, 2
    pos0 = 4 * T_total - 1 - steps - 1
    max_seq = 4 * T_total + 16
    args, full, inputs = make_case(3, 1, T_total, W, k, steps, pos0)
    want, want_idx, want_score = oracle_outputs(args, full, inputs, pos0, max_seq, with_scores=True)
    one, sel1 = _run_split(args, full, inputs, 1, T_total, pos0, max_seq, cuda_dev, 1)
    for G in (1, 2, 8):
        outg, selg = (one, sel1) if G == 1 else _run_split(args, full, inputs, G, T_total, pos0, max_seq,
                                                          cuda_dev, 1)
        for s in range(steps):
            t_active = (pos0 + s + 1) // 4
            got = torch.where(selg[s] >= 0, selg[s] + W, torch.full_like(selg[s], -1))
            assert_topk_sets(got, want_idx[s][:, W:], masked_scores(want_score[s], t_active), W,
                             what=f"G={G} step {s}")
            assert set(sel1[s][0].tolist()) == set(selg[s][0].tolist()), (G, s)
            for g in range(G):
                assert torch.allclose(outg[s][g].float(), want[s].float(), rtol=2e-2, atol=2e-2), (G, s, g)


def test_single_shard_path_writes_final_output(cuda_dev):
    """World of one through SeqSplitPath: the attention writes the final
    output directly (no partial exchange, no combine) and matches the oracle."""
    from dsv4attn.dist import SeqShard, SeqSplitPath
    T_total, W, k, steps = 4096, 128, 512, 4
    pos0 = 4 * T_total - 1 - steps - 3
    max_seq = 4 * T_total + 64
    args, full, inputs = make_case(55, 1, T_total, W, k, steps, pos0)
    want, _ = oracle_outputs(args, full, inputs, pos0, max_seq)
    shard = SeqShard(args, 1, T_total, 0, 1, cuda_dev, k=k, max_seq_len=max_seq)
    load_shard(shard, full)
    shard.set_positions(pos0)
    path = SeqSplitPath(shard)
    for s, x in enumerate(inputs):
        xd = type(x)(*[t.to(cuda_dev) for t in x.tensors()])
        out = torch.empty(1, args.n_heads, args.head_dim, dtype=BF16, device=cuda_dev)
        path.step([xd], [out])
        torch.cuda.synchronize()
        assert torch.allclose(out.cpu().float(), want[s].float(), rtol=2e-2, atol=2e-2), s
    assert int(shard.status.item()) == 0
