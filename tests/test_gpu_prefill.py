"""GPU parity of the multi-token (prefill-chunk) path (BASELINE config 4
shape family): per-token causal T_active, dense indexer scores with a
shared key cache, per-token top-k and sink attention over W + k rows.

Bars: indexer scores rtol 1e-3 (fp32 accumulation of the same bf16
inputs); top-k sets equal except near-ties (relative gap < 1e-3);
attention outputs rtol/atol 2e-2 of the fp32 oracle.  The full config-4
size (4096 tokens x 32768 entries, top-2048) is checked on a sample of
tokens against the oracle run on those tokens alone."""

import pytest
import torch

import oracle.path as ref

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
H, D, Hi, Di = 64, 512, 64, 128


def _case(seed, S, T, n_hist, base):
    g = torch.Generator().manual_seed(seed)
    n_raw = n_hist + S
    return dict(
        q=torch.randn(S, H, D, generator=g).to(BF16),
        kv=torch.randn(n_raw + T, D, generator=g).to(BF16),
        iq=torch.randn(S, Hi, Di, generator=g).to(BF16),
        ikeys=torch.randn(T, Di, generator=g).to(BF16),
        iw=0.02 * torch.randn(S, Hi, generator=g),
        sink=torch.randn(H, generator=g), n_raw=n_raw)


def _run(dev, c, S, T, k, base, n_hist):
    from dsv4attn.prefill import PrefillChunk
    from dsv4attn.tables import PathArgs
    ch = PrefillChunk(PathArgs(index_topk=k), S, T, dev)
    o = ch.run(c["q"].to(dev), c["kv"].to(dev), c["n_raw"], c["iq"].to(dev), c["ikeys"].to(dev),
               c["iw"].to(dev), c["sink"].to(dev), base, n_hist, T)
    torch.cuda.synchronize()
    assert int(ch.status.item()) == 0
    return ch, o.cpu()


def _sets_match(got_idx, want_idx, score, n_raw, W):
    for s in range(got_idx.shape[0]):
        g = set(int(v) for v in got_idx[s, W:] if v >= 0)
        w = set(int(v) for v in want_idx[s, W:] if v >= 0)
        if g == w:
            continue
        kth = min(float(score[s, v - n_raw]) for v in w)
        for v in g ^ w:
            assert abs(float(score[s, v - n_raw]) - kth) <= 1e-3 * max(abs(kth), 1e-6), (s, v)


@pytest.mark.parametrize("S,T,k,base,n_hist", [
    (64, 1024, 256, 4 * 1024 - 64, 127),   # full visibility, selection among ~1000
    (48, 512, 64, 200, 100),               # t_active 50..62 < k (invalid slots), short history
    (32, 2048, 512, 4000, 0),              # no raw history: the first windows are partly empty
    (30, 700, 128, 2700, 127),             # S not a multiple of 4: the per-token (decode) kernel, shared keys
])
def test_prefill_chunk_matches_oracle(cuda_dev, S, T, k, base, n_hist):
    c = _case(S + T, S, T, n_hist, base)
    ch, o = _run(cuda_dev, c, S, T, k, base, n_hist)
    want, widx = ref.prefill_chunk(c["q"], c["kv"], c["n_raw"], c["iq"], c["ikeys"], c["iw"], c["sink"], base,
                                   n_hist, T, k)
    gidx = ch.idx.cpu()
    assert torch.equal(gidx[:, :128], widx[:, :128])
    score = (torch.einsum("shd,td->sht", c["iq"].float(), c["ikeys"].float()).relu()
             * c["iw"].unsqueeze(-1)).sum(1)
    ta = torch.tensor([min(T, (base + s + 1) // 4) for s in range(S)])
    assert torch.equal(ch.t_active.cpu(), ta.to(torch.int32))
    gs = ch.score.cpu()
    for s in range(S):
        t = int(ta[s])
        assert torch.allclose(gs[s, :t], score[s, :t], rtol=1e-3, atol=1e-4)
    _sets_match(gidx, widx, score, c["n_raw"], 128)
    assert torch.allclose(o.float(), want.float(), rtol=2e-2, atol=2e-2)


def test_prefill_config4_size_sampled(cuda_dev):
    S, T, k, n_hist = 4096, 32768, 2048, 127
    base = 131072 - S
    c = _case(4, S, T, n_hist, base)
    ch, o = _run(cuda_dev, c, S, T, k, base, n_hist)
    sample = [0, 1, 777, 2048, 4095]
    want, widx = ref.prefill_chunk(c["q"][sample], c["kv"], c["n_raw"], c["iq"][sample], c["ikeys"],
                                   c["iw"][sample], c["sink"], base, n_hist, T, k, rows=sample)
    gidx = ch.idx.cpu()[sample]
    score = (torch.einsum("shd,td->sht", c["iq"][sample].float(), c["ikeys"].float()).relu()
             * c["iw"][sample].unsqueeze(-1)).sum(1)
    _sets_match(gidx, widx, score, c["n_raw"], 128)
    assert torch.allclose(o[sample].float(), want.float(), rtol=2e-2, atol=2e-2)
