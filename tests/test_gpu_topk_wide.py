"""GPU parity of the multi-CTA top-k (dsa_topk_wide) for few long rows:
the selected set must equal the CPU oracle's top-k set (inference.py:5823-5851)
except at near-ties, and the per-row kernel's exact set (same masking,
validity and lower-position tie rule), output in ascending position order,
including adversarial score distributions and the candidate-merge mode."""

import pytest
import torch

import oracle as O
from parity import assert_topk_sets, masked_scores

pytestmark = pytest.mark.gpu


def _scores(kind, B, T, g):
    if kind == "normal":
        return torch.randn(B, T, generator=g)
    if kind == "equal":
        return torch.full((B, T), 0.5)
    if kind == "few":
        return torch.randint(0, 3, (B, T), generator=g).float()
    if kind == "quantized":
        return (torch.randn(B, T, generator=g) * 4).round() / 4
    if kind == "neg_inf":
        s = torch.randn(B, T, generator=g)
        s[:, ::3] = float("-inf")
        return s
    if kind == "tiny_range":
        return 1.0 + torch.rand(B, T, generator=g) * 1e-6
    raise ValueError(kind)


def _ref(score, ta, k, win, mask_mode, dev):
    from dsv4attn import ops
    out = ops.indexer_topk(score, ta, k, win, sort_desc=False, mask_mode=mask_mode)
    return out


@pytest.mark.parametrize("kind", ["normal", "equal", "few", "quantized", "neg_inf", "tiny_range"])
@pytest.mark.parametrize("B,T,k,mask_mode", [(1, 65536, 2048, 1), (2, 8192, 2048, 0), (1, 16384, 2048, 1),
                                              (3, 1000, 1000, 0), (1, 4096, 7, 1), (2, 300, 17, 1), (1, 1, 1, 0),
                                              (1, 100000, 2048, 1)])
def test_topk_wide_equals_per_row_kernel(cuda_dev, kind, B, T, k, mask_mode):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(T + k + B)
    s = _scores(kind, B, T, g).to(cuda_dev)
    ta = torch.tensor([T - (T // 5) * (b % 2) for b in range(B)], dtype=torch.int32, device=cuda_dev)
    win = 128
    st = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    osc = torch.empty(B, k, device=cuda_dev)
    got = ops.topk_wide(s, k, win, t_active=ta, mask_mode=mask_mode, out_score=osc, status=st)
    want = _ref(s, ta, k, win, mask_mode, cuda_dev)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    s_cpu, ta_cpu = s.cpu(), ta.cpu()
    assert_topk_sets(got.cpu(), O.indexer_topk(s_cpu, ta_cpu, k, win), masked_scores(s_cpu, ta_cpu), win,
                     what=f"{kind} vs oracle")
    for b in range(B):
        gv = got[b].cpu()
        wv = want[b].cpu()
        assert sorted(gv.tolist()) == sorted(wv.tolist()), (kind, b)
        valid = gv[gv >= 0]
        assert torch.all(valid[1:] > valid[:-1]), "valid outputs must ascend by position"


def test_topk_wide_repeated_calls_reuse_workspace(cuda_dev):
    """The workspace is left zeroed, so back-to-back calls of different
    shapes on one workspace stay exact."""
    from dsv4attn import ops
    ws = ops.WideTopkWorkspace(cuda_dev)
    g = torch.Generator().manual_seed(1)
    for T, B, k in ((65536, 1, 2048), (3000, 2, 100), (100000, 1, 2048), (16384, 1, 2048), (100000, 1, 64),
                    (65536, 1, 2048)):
        s = torch.randn(B, T, generator=g).to(cuda_dev)
        got = ops.topk_wide(s, k, 0, T=T, mask_mode=1, ws=ws)
        ta = torch.full((B,), T, dtype=torch.int32, device=cuda_dev)
        want = ops.indexer_topk(s, ta, k, 0, sort_desc=False, mask_mode=1)
        torch.cuda.synchronize()
        assert torch.equal(got.sort(dim=1).values, want.sort(dim=1).values)


def test_topk_wide_merge_mode_equals_topk_merge(cuda_dev):
    """Candidate merge: 8 shards x 2048 (score, global position) in
    ascending position order, some empty (-1); same set as dsa_topk_merge."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(5)
    G, kc, k = 8, 2048, 2048
    per = 8192
    ids = []
    for r in range(G):
        pos = torch.randperm(per, generator=g)[:kc].sort().values + r * per
        ids.append(pos)
    ci = torch.cat(ids).to(torch.int32).view(1, -1)
    cs = torch.randn(1, G * kc, generator=g)
    ci[0, 5::97] = -1
    cs[0, 5::97] = float("-inf")
    ci, cs = ci.to(cuda_dev), cs.to(cuda_dev)
    got = ops.topk_wide(cs, k, 128, ids=ci, mask_mode=0)
    want = ops.topk_merge(cs, ci, k, 128)
    torch.cuda.synchronize()
    assert sorted(got[0].tolist()) == sorted(want[0].tolist())


def test_topk_wide_segmented_rows_equal_contiguous(cuda_dev):
    """A row read as G segments seg_stride apart (the rank-major all-gather
    of [scores | ids] lists) selects what the contiguous row selects."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(9)
    G, B, kc, k = 4, 2, 512, 700
    blocks = []
    sc = torch.randn(G, B, kc, generator=g)
    ix = torch.arange(G * kc, dtype=torch.int32).view(G, 1, kc).expand(G, B, kc).contiguous()
    for r in range(G):
        blocks.append(torch.cat([sc[r].reshape(-1).view(torch.int32), ix[r].reshape(-1)]))
    flat = torch.stack(blocks).to(cuda_dev).view(-1)
    got = ops.topk_wide(flat.view(torch.float32), k, 3, ids=flat[B * kc:], mask_mode=0, seg_len=kc,
                        seg_stride=2 * B * kc, B=B, T=G * kc, ld_score=kc)
    cs = sc.permute(1, 0, 2).reshape(B, G * kc).to(cuda_dev)
    ci = ix.permute(1, 0, 2).reshape(B, G * kc).to(cuda_dev)
    want = ops.topk_wide(cs, k, 3, ids=ci, mask_mode=0)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
