"""GPU parity: attn.topk (window indices, indexer score, masked top-k,
candidate merge) and attn.sparse (gather + sink-softmax attention) against
the CPU oracle.

Bars: top-k index sets identical except at documented
near-ties - a position counts as a near-tie when its oracle score is within
relative 1e-3 of the k-th oracle score; indexer scores within rtol 1e-3;
attention outputs within rtol 2e-2 / atol 2e-2 of the fp32 oracle."""

import pytest
import torch

import oracle as O
from parity import NEAR_TIE_REL, assert_topk_sets  # noqa: F401

pytestmark = pytest.mark.gpu


def rel_err(got, want):
    g, w = got.float(), want.float()
    return float((g - w).norm() / w.norm().clamp_min(1e-30))


ATTN_REL = 1e-2   # relative Frobenius error bound for the attention outputs


def masked_scores(score, t_active):
    T = score.shape[1]
    ta = torch.as_tensor(t_active).reshape(-1, 1)
    return score - 1e4 * (torch.arange(T).unsqueeze(0) >= ta).float()


@pytest.mark.parametrize("pos", [0, 5, 127, 128, 200, 4095])
def test_window_indices(cuda_dev, pos):
    from dsv4attn import ops
    got = ops.window_indices(torch.tensor([pos, pos + 1], dtype=torch.int32, device=cuda_dev), 128).cpu()
    assert torch.equal(got[0], O.window_indices(pos, 128))
    assert torch.equal(got[1], O.window_indices(pos + 1, 128))


@pytest.mark.parametrize("B,T", [(1, 1024), (3, 1000), (2, 77), (64, 8192)])
def test_indexer_score(cuda_dev, B, T):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B * 100 + T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T + 5, 128, generator=g).to(torch.bfloat16)
    w = 0.02 * torch.randn(B, 64, generator=g)
    want = O.indexer_score(q, k[:, :T], w)
    got = ops.indexer_score(q.to(cuda_dev), k.to(cuda_dev), w.to(cuda_dev), T).cpu()
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3 * float(want.abs().max()))


@pytest.mark.parametrize("B,T,tv_lo", [(64, 9216, 8000), (3, 1000, 0), (300, 700, 1)])
def test_indexer_score_keys_ready_identical(cuda_dev, B, T, tv_lo):
    """DSA_KEYS_READY (first key tiles requested before the launch wait)
    gives bit-identical scores, entries at and past t_valid untouched,
    also when q and w are rewritten right before the call."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    k = torch.randn(B, T, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    w = (0.02 * torch.randn(B, 64, generator=g)).to(cuda_dev)
    tv = torch.randint(tv_lo, T + 1, (B,), generator=g, dtype=torch.int32).to(cuda_dev)
    want = torch.full((B, T), 7.0, device=cuda_dev)
    ops.indexer_score(q, k, w, T, out=want, t_valid=tv)
    q2, w2 = torch.zeros_like(q), torch.zeros_like(w)
    for _ in range(2):
        got = torch.full((B, T), 7.0, device=cuda_dev)
        q2.copy_(q)
        w2.copy_(w)
        ops.indexer_score(q2, k, w2, T, out=got, t_valid=tv, keys_ready=True)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def test_indexer_score_t_valid(cuda_dev):
    from dsv4attn import ops
    B, T = 2, 512
    q = torch.randn(B, 64, 128).to(torch.bfloat16)
    k = torch.randn(B, T, 128).to(torch.bfloat16)
    w = 0.02 * torch.randn(B, 64)
    out = torch.full((B, T), 123.0, device=cuda_dev)
    tv = torch.tensor([100, 0], dtype=torch.int32, device=cuda_dev)
    ops.indexer_score(q.to(cuda_dev), k.to(cuda_dev), w.to(cuda_dev), T, out=out, t_valid=tv)
    want = O.indexer_score(q, k, w)
    o = out.cpu()
    torch.testing.assert_close(o[0, :100], want[0, :100], rtol=1e-3, atol=1e-4)
    assert (o[0, 100:] == 123.0).all() and (o[1] == 123.0).all()


@pytest.mark.parametrize("B,T,zero_frac", [(300, 700, 0.2), (4500, 64, 0.2), (7, 1000, 0.9)])
def test_indexer_score_ragged_t_valid(cuda_dev, B, T, zero_frac):
    # ragged live lengths: empty sequences, partial last tiles, t_valid past T
    # (clamped); 4500 sequences take the all-items walk, the others the
    # live-tile split, and (7, 1000) leaves most CTAs without work
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, T, 128, generator=g).to(torch.bfloat16)
    w = 0.02 * torch.randn(B, 64, generator=g)
    tv = torch.randint(0, T + 41, (B,), generator=g, dtype=torch.int32)
    tv[torch.rand(B, generator=g) < zero_frac] = 0
    out = torch.full((B, T), 123.0, device=cuda_dev)
    ops.indexer_score(q.to(cuda_dev), k.to(cuda_dev), w.to(cuda_dev), T, out=out, t_valid=tv.to(cuda_dev))
    want = O.indexer_score(q, k, w)
    o = out.cpu()
    lim = tv.clamp(max=T)
    live = torch.arange(T)[None, :] < lim[:, None]
    torch.testing.assert_close(o[live], want[live], rtol=1e-3, atol=1e-3 * float(want.abs().max()))
    assert (o[~live] == 123.0).all()


@pytest.mark.parametrize("B,T,k", [(64, 9216, 2048), (2, 20000, 512)])
def test_indexer_topk_newest_recomputes_last_row(cuda_dev, B, T, k):
    # the decode step scores rows [0, t_active - 1) while the compressor
    # writes the newest row; the top-k must recompute that row's score (its
    # stored value is planted wrong here) and select what scoring every row
    # first selects; T = 20000 takes the two-level (chunk + merge) path
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, T, 128, generator=g).to(torch.bfloat16)
    w = 0.02 * torch.randn(B, 64, generator=g)
    ta = torch.randint(k, T + 1, (B,), generator=g, dtype=torch.int32)
    ta[0], ta[-1] = T, k
    W = 128
    qd, kd, wd, tad = q.to(cuda_dev), kc.to(cuda_dev), w.to(cuda_dev), ta.to(cuda_dev)
    score = torch.zeros(B, T, device=cuda_dev)
    ops.indexer_score(qd, kd, wd, T, out=score, t_valid=tad - 1)
    score[torch.arange(B, device=cuda_dev), (tad - 1).long()] = 1e6
    got = ops.indexer_topk(score, tad, k, W, T=T, mask_mode=1, refresh=(qd, kd, wd)).cpu()
    full = O.indexer_score(q, kc, w)
    masked = full.masked_fill(torch.arange(T)[None, :] >= ta[:, None], float("-inf"))
    want = torch.topk(masked, k, dim=1).indices.int() + W
    assert_topk_sets(got, want, masked, W)


def test_topk_reference_case(cuda_dev):
    # T_PAD 128, bucket 128, k 64, T_active 50 (test_lk_d_topk.py:42-46, 219-224)
    from dsv4attn import ops
    torch.manual_seed(0)
    score = torch.randn(1, 128).to(torch.bfloat16).float()
    want = O.indexer_topk(score, 50, 64, 128)
    for sort_desc in (False, True):
        got = ops.indexer_topk(score.to(cuda_dev), torch.tensor([50], dtype=torch.int32, device=cuda_dev), 64, 128,
                               sort_desc=sort_desc).cpu()
        assert set(got[0].tolist()) == set(want[0].tolist())
        assert int((got[0] == -1).sum()) == 14
        if sort_desc:
            # descending masked score, the -1 sentinels last (reference sorted=True)
            valid = got[0][got[0] >= 0] - 128
            vals = score[0, valid.long()]
            assert (vals[:-1] >= vals[1:]).all()
            assert (got[0, :50] >= 0).all() and (got[0, 50:] == -1).all()


def test_topk_one_hot_and_ties(cuda_dev):
    from dsv4attn import ops
    score = torch.zeros(2, 300)
    score[0, 17] = 5.0
    score[1, :] = 1.0                        # all tied: lowest indices win
    ta = torch.tensor([300, 300], dtype=torch.int32, device=cuda_dev)
    got = ops.indexer_topk(score.to(cuda_dev), ta, 10, 0).cpu()
    assert 17 in got[0].tolist()
    assert sorted(got[1].tolist()) == list(range(10))


@pytest.mark.parametrize("B,T,k,ta", [(1, 1024, 512, 1024), (4, 1024, 512, 700), (64, 8192, 2048, 8192),
                                      (2, 8192, 2048, 1000), (1, 65536, 2048, 65536), (2, 40000, 2048, 30000)])
def test_topk_random_sets(cuda_dev, B, T, k, ta):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(T + k)
    score = torch.randn(B, T, generator=g)
    tact = torch.full((B,), ta, dtype=torch.int32)
    want = O.indexer_topk(score, tact, k, 128)
    got = ops.indexer_topk(score.to(cuda_dev), tact.to(cuda_dev), k, 128).cpu()
    assert_topk_sets(got, want, masked_scores(score, tact), 128)
    assert int((got == -1).sum()) == int((want == -1).sum())


def _exact_topk_rows(score, tact, k, win):
    """Deterministic top-k with -inf masking (mask_mode 1): every position
    above the k-th value, then the lowest positions equal to it; -1 for picks
    that are masked."""
    out = []
    for b in range(score.shape[0]):
        row = score[b].clone()
        row[int(tact[b]):] = float("-inf")
        thr = torch.sort(row, descending=True).values[k - 1]
        above = torch.nonzero(row > thr).flatten().tolist()
        eq = torch.nonzero(row == thr).flatten().tolist()
        pick = above + eq[:k - len(above)]
        out.append(sorted((i + win) if row[i] >= -1000 else -1 for i in pick))
    return out


@pytest.mark.parametrize("kind", ["quantized", "cluster", "lognormal", "floor", "equal", "few", "prod"])
def test_topk_exact_distributions(cuda_dev, kind):
    """Exact sets (ties to the lowest position) on score distributions that
    drive every branch of the selection: quantized and clustered values
    (several levels, exact-value exit), very wide dynamic range, thresholds at
    the masked floor, all-equal rows, short rows, and the production shape."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(sum(map(ord, kind)))
    B, T, k, ta = 3, 9216, 2048, 8192
    if kind == "quantized":
        score = torch.randint(0, 40, (B, T), generator=g).float() * 0.25
    elif kind == "cluster":
        score = torch.ones(B, T)
        hot = torch.rand(B, T, generator=g) < 0.01
        score[hot] = 1.0 + torch.rand(int(hot.sum()), generator=g)
        score[:, ::7] = 1.0 - 1e-7 * torch.arange(0, T, 7).float()
    elif kind == "lognormal":
        score = torch.exp(20.0 * torch.randn(B, T, generator=g))
    elif kind == "floor":
        score = torch.randn(B, T, generator=g)
        ta = 1500  # fewer live positions than k
    elif kind == "equal":
        score = torch.full((B, T), -3.5)
    elif kind == "few":
        T, k, ta = 300, 64, 250
        score = torch.randn(B, T, generator=g)
    else:
        B = 64
        score = 0.02 * torch.randn(B, T, generator=g).abs()
    tact = torch.full((B,), ta, dtype=torch.int32)
    got = ops.indexer_topk(score.to(cuda_dev), tact.to(cuda_dev), k, 128, T=T, mask_mode=1).cpu()
    want = _exact_topk_rows(score, tact, k, 128)
    for b in range(B):
        assert sorted(got[b].tolist()) == want[b], f"{kind} row {b}"


def test_topk_mask_mode_exclusion_equivalent(cuda_dev):
    from dsv4attn import ops
    B, T, k = 3, 4096, 512
    score = torch.randn(B, T)
    tact = torch.tensor([4096, 300, 0], dtype=torch.int32)
    a = ops.indexer_topk(score.to(cuda_dev), tact.to(cuda_dev), k, 128, mask_mode=0).cpu()
    poisoned = score.clone()
    for b in range(B):
        poisoned[b, int(tact[b]):] = float("nan")   # never read in mask_mode 1
    bm = ops.indexer_topk(poisoned.to(cuda_dev), tact.to(cuda_dev), k, 128, mask_mode=1).cpu()
    for b in range(B):
        assert set(a[b].tolist()) == set(bm[b].tolist())


def test_topk_merge_equals_global(cuda_dev):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(11)
    T, G, k = 65536, 8, 2048
    score = torch.randn(1, T, generator=g)
    want = O.indexer_topk(score, T, k, 128)
    cs, ci = [], []
    for r in range(G):
        sub = score[:, r * T // G:(r + 1) * T // G]
        v, i = torch.topk(sub, k)
        cs.append(v)
        ci.append((i + r * T // G).to(torch.int32))
    got = ops.topk_merge(torch.cat(cs, 1).to(cuda_dev), torch.cat(ci, 1).to(cuda_dev), k, 128).cpu()
    assert_topk_sets(got, want, score, 128)


# --------------------------------------------------------------- attention

def _attn_case(B, S, N, K, frac_masked=0.1, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, 64, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, N, 512, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, N, (B, S, K), generator=g, dtype=torch.int32)
    idx[torch.rand(B, S, K, generator=g) < frac_masked] = -1
    sink = torch.randn(64, generator=g)
    return q, kv, idx, sink


@pytest.mark.parametrize("B,S,N,K", [(1, 1, 4224, 640), (2, 1, 1000, 200), (64, 1, 2048, 2176), (1, 1, 70000, 2176),
                                     (2, 3, 600, 130), (1, 1, 300, 17)])
def test_sparse_attn_matches_oracle(cuda_dev, B, S, N, K):
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(B, S, N, K, seed=N + K)
    scale = 512 ** -0.5
    want = O.sparse_attn(q, kv, idx, sink, scale)
    lse = torch.empty(B * S, 64, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    got = ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), scale, lse=lse,
                          status=status).cpu()
    assert int(status.item()) == 0, f"device status {int(status.item())} (1 = bad index, 2 = wait timeout)"
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
    assert rel_err(got, want) < ATTN_REL, rel_err(got, want)
    # log-sum-exp of [z | sink] per head
    qf, kvf = q.float().reshape(B * S, 64, 512), kv.float()
    for mrow in (0, B * S - 1):
        bb = mrow // S
        ids = idx.reshape(B * S, K)[mrow]
        z = (qf[mrow] @ kvf[bb, ids.clamp_min(0).long()].T) * scale
        z[:, ids < 0] = float("-inf")
        ref = torch.logsumexp(torch.cat([z, sink.unsqueeze(1)], 1), 1)
        torch.testing.assert_close(lse[mrow].cpu(), ref, rtol=1e-3, atol=1e-3)


def test_sparse_attn_all_masked_and_single_index(cuda_dev):
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(1, 1, 64, 128, seed=5)
    idx[:] = -1
    got = ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), 0.05).cpu()
    assert (got == 0).all()
    idx[0, 0, 77] = 9
    want = O.sparse_attn(q, kv, idx, sink, 0.05)
    got = ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), 0.05).cpu()
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
    assert rel_err(got, want) < ATTN_REL


def test_sparse_attn_out_of_range_index_flags_status(cuda_dev):
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(1, 1, 100, 64, seed=6)
    idx[0, 0, 3] = 100        # == kv_rows: clamped and reported, never read out of bounds
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), 0.05, status=status)
    assert int(status.item()) != 0


def test_sparse_attn_partial_combine_equals_full(cuda_dev):
    """Sequence-split building block: partials over disjoint index subsets
    merged by lse_combine (sink once) equal the unsplit attention."""
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(1, 1, 5000, 2176, seed=8)
    qd, kvd, sd = q.to(cuda_dev), kv.to(cuda_dev), sink.to(cuda_dev)
    full = ops.sparse_attn(qd, kvd, idx.to(cuda_dev), sd, 0.044)
    parts = []
    G = 4
    for r in range(G):
        sub = idx.clone()
        keep = (sub >= r * 1250) & (sub < (r + 1) * 1250)
        sub[~keep] = -1
        parts.append(ops.sparse_attn_partial(qd, kvd, sub.to(cuda_dev), 0.044))
    ml = torch.stack([p[0] for p in parts])
    po = torch.stack([p[1] for p in parts])
    comb = ops.lse_combine(ml, po, sd).view(1, 1, 64, 512)
    torch.testing.assert_close(comb.float().cpu(), full.float().cpu(), rtol=2e-2, atol=2e-2)
    want = O.sparse_attn(q, kv, idx, sink, 0.044)
    torch.testing.assert_close(comb.float().cpu(), want.float(), rtol=2e-2, atol=2e-2)
    assert rel_err(comb.cpu(), want) < ATTN_REL and rel_err(full.cpu(), want) < ATTN_REL


def test_sparse_attn_peaked_softmax(cuda_dev):
    """Scaled-up queries make the softmax peaked (outputs O(1)) and exercise the
    lazy-rescale path many times per split."""
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(4, 1, 3000, 2176, frac_masked=0.05, seed=21)
    q = (q.float() * 6).to(torch.bfloat16)
    # sorted descending-ish scores so the running max keeps moving up
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    want = O.sparse_attn(q, kv, idx, sink, 512 ** -0.5)
    got = ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), 512 ** -0.5,
                          status=status).cpu()
    assert int(status.item()) == 0
    assert float(want.float().abs().max()) > 0.5
    assert rel_err(got, want) < ATTN_REL, rel_err(got, want)


@pytest.mark.parametrize("B,N,K,lead", [(64, 2048, 2176, 128), (1, 70000, 2176, 128), (4, 4224, 640, 128),
                                        (3, 900, 256, 64), (2, 600, 130, 128)])
def test_sparse_attn_lead_tiles_match_oracle(cuda_dev, B, N, K, lead):
    """dsa_sparse_attn_ex with DSA_LEAD_READY (each key split takes one
    window tile first, requested before the dependency wait): the same
    output and log-sum-exp as the oracle, including a lead tile whose
    entries are partly masked, and shapes where the lead mapping does not
    apply (fewer splits than lead tiles) and the plain mapping runs."""
    from dsv4attn import ops
    q, kv, idx, sink = _attn_case(B, 1, N, K, seed=3 * N + K)
    idx[:, :, 5] = -1
    scale = 512 ** -0.5
    want = O.sparse_attn(q, kv, idx, sink, scale)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    lse = torch.empty(B, 64, device=cuda_dev)
    lse0 = torch.empty(B, 64, device=cuda_dev)
    qd, kvd, idd, sd = q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev)
    got = ops.sparse_attn(qd, kvd, idd, sd, scale, lse=lse, status=status, lead_cols=lead, lead_ready=True).cpu()
    plain = ops.sparse_attn(qd, kvd, idd, sd, scale, lse=lse0).cpu()
    assert int(status.item()) == 0
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
    assert rel_err(got, want) < ATTN_REL
    # the two differ by the bf16 rounding of differently composed split partials
    torch.testing.assert_close(got.float(), plain.float(), rtol=2e-2, atol=4e-3)
    torch.testing.assert_close(lse.cpu(), lse0.cpu(), rtol=1e-4, atol=1e-4)


def test_sparse_attn_ex_rejects_bad_lead(cuda_dev):
    from dsv4attn import _lib
    q, kv, idx, sink = (t.to(cuda_dev) for t in _attn_case(1, 1, 300, 64, seed=1))
    out = torch.empty_like(q)
    L = _lib.lib()
    rc = L.dsa_sparse_attn_ex(q.data_ptr(), kv.data_ptr(), 300 * 512, 300, idx.data_ptr(), 64, sink.data_ptr(),
                              out.data_ptr(), None, 1, 1, 64, 512, 64, 0.05, None, 0, 128, 1, None, None)
    assert rc != 0 and "lead_cols" in _lib.last_error()


@pytest.mark.parametrize("B", [24, 80])
@pytest.mark.parametrize("kind", ["gauss", "ties", "const_rows", "wide", "nan", "short"])
def test_topk_position_order_equals_sorted_selection(cuda_dev, kind, B):
    # the position-order top-k (one row per CTA, its own first level) and
    # the sorted top-k (the general select) pick exactly the same indices:
    # the k largest, ties to the lowest positions -- no near-tie allowance.
    # Rows the position-order kernels hand to the general select (constant
    # rows, huge ranges, NaN, fewer than k live entries) included; 24 rows
    # run two CTAs per row (a cluster pair), 80 rows one CTA per row.
    from dsv4attn import ops
    T, k, W = 9216, 2048, 128
    g = torch.Generator().manual_seed(hash(kind) % 1000)
    s = torch.randn(B, T, generator=g) * (0.8 + torch.rand(B, 1, generator=g)) + 3 * (torch.rand(B, 1, generator=g) - .5)
    if kind == "ties":
        s = torch.floor(s * 4) / 4
    elif kind == "const_rows":
        s[::3] = 1.0
    elif kind == "wide":
        s[:, ::7] = 1e30
    elif kind == "nan":
        s[::5, 17] = float("nan")
    ta = torch.randint(k, T + 1, (B,), generator=g, dtype=torch.int32)
    if kind == "short":
        ta = torch.randint(1, k, (B,), generator=g, dtype=torch.int32)
    sd, tad = s.to(cuda_dev), ta.to(cuda_dev)
    pos_order = ops.indexer_topk(sd, tad, k, W, mask_mode=1).cpu()
    srt = ops.indexer_topk(sd, tad, k, W, mask_mode=1, sort_desc=True).cpu()
    for b in range(B):
        a = sorted(int(v) for v in pos_order[b] if v >= 0)
        c = sorted(int(v) for v in srt[b] if v >= 0)
        assert a == c, f"{kind} row {b}"
        assert int((pos_order[b] < 0).sum()) == int((srt[b] < 0).sum())


@pytest.mark.parametrize("B,T", [(64, 9216), (3, 20000), (5, 640)])
def test_indexer_score_newest_matches_refresh(cuda_dev, B, T):
    # the newest live row's score written by its own kernel (the decode
    # step's side branch) is the value the top-k's refresh recomputes: the
    # plain top-k then selects exactly what the refresh top-k selects; only
    # entry t_active - 1 of each row is written
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + T)
    k = min(512, T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    kc = torch.randn(B, T, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    w = (0.02 * torch.randn(B, 64, generator=g)).to(cuda_dev)
    ta = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32)
    ta[0] = T
    tad = ta.to(cuda_dev)
    score = torch.full((B, T), 123.0, device=cuda_dev)
    ops.indexer_score(q, kc, w, T, out=score, t_valid=tad - 1)
    before = score.clone()
    ops.indexer_score_newest(q, kc, w, tad, T, out=score)
    ws = ops.Workspace(cuda_dev, int(ops.lib().dsa_indexer_topk_workspace_size(B, T, k)) or 16)
    plain = ops.indexer_topk(score, tad, k, 128, T=T, mask_mode=1, ws=ws)
    refreshed = ops.indexer_topk(before, tad, k, 128, T=T, mask_mode=1, ws=ws, refresh=(q, kc, w))
    torch.cuda.synchronize()
    assert torch.equal(plain.cpu(), refreshed.cpu())
    changed = (score != before).cpu()
    rows = torch.arange(B)
    assert bool(changed[rows, (ta - 1).long()].all())
    changed[rows, (ta - 1).long()] = False
    assert not bool(changed.any())
    want = O.indexer_score(q.cpu(), kc.cpu(), w.cpu())
    got = score.cpu()[rows, (ta - 1).long()]
    torch.testing.assert_close(got, want[rows, (ta - 1).long()], rtol=1e-3,
                               atol=1e-3 * float(want.abs().max()))


def test_sparse_attn_pair_combine_deterministic(cuda_dev):
    # 64 query rows x 2176 keys run as pairs of key splits that finish the
    # row between them over distributed shared memory: repeated calls give
    # identical bits, and every row matches the oracle
    from dsv4attn import ops
    B, N, K = 64, 2400, 2176
    q, kv, idx, sink = _attn_case(B, 1, N, K, seed=77)
    idx = idx.clone()
    idx.view(B, K)[::7, -300:] = -1
    qd, kvd, idd, sd = q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev)
    a = ops.sparse_attn(qd, kvd, idd, sd, 512 ** -0.5).cpu()
    b = ops.sparse_attn(qd, kvd, idd, sd, 512 ** -0.5).cpu()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    want = O.sparse_attn(q, kv, idx, sink, 512 ** -0.5)
    assert rel_err(a, want) < ATTN_REL


@pytest.mark.parametrize("B,T,keys_ready", [(64, 9216, True), (64, 9216, False), (7, 3000, True), (130, 640, False)])
def test_indexer_score_dynamic_split_equals_static(cuda_dev, B, T, keys_ready):
    # claiming items from a counter changes which CTA scores which tile, not
    # a score: equal bits to the static split, over repeated calls (the
    # counters come back to zero) and ragged t_valid
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + T)
    q = torch.randn(B, 64, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    k = torch.randn(B, T, 128, generator=g).to(torch.bfloat16).to(cuda_dev)
    w = (0.02 * torch.randn(B, 64, generator=g)).to(cuda_dev)
    tv = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    tv[0] = T
    tvd = tv.to(cuda_dev)
    ctr = torch.zeros(2, dtype=torch.int32, device=cuda_dev)
    want = torch.full((B, T), 5.0, device=cuda_dev)
    ops.indexer_score(q, k, w, T, out=want, t_valid=tvd)
    for rep in range(3):
        got = torch.full((B, T), 5.0, device=cuda_dev)
        ops.indexer_score(q, k, w, T, out=got, t_valid=tvd, keys_ready=keys_ready, counters=ctr)
        torch.cuda.synchronize()
        assert torch.equal(got.cpu(), want.cpu()), f"call {rep}"
        assert ctr.cpu().tolist() == [0, 0]
