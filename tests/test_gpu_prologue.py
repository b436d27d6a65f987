"""The decode layer's prologue (dsa_layer_prologue: the indexer compressor
and the newest row's score, the window-ring KV write, the window indices and
the attention compressor in one launch) against the five separate calls it
replaces, bit for bit, over consecutive decode steps that include emit and
non-emit positions, with and without DSA_BESIDE_PREVIOUS (run beside the
previous kernel: here an indexer score that covers the rows before the
newest, as in the decode step)."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _state(B, D, Di, W, T, r, g, dev):
    def rnd(*shape, dtype=torch.float32, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dtype).to(dev)
    s = {
        "kv_cache": rnd(B, W + T, D, dtype=BF), "idx_cache": rnd(B, T, Di, dtype=BF),
        "kv_state": rnd(B, 2 * r, 2 * D), "sc_state": rnd(B, 2 * r, 2 * D),
        "ikv_state": rnd(B, 2 * r, 2 * Di), "isc_state": rnd(B, 2 * r, 2 * Di),
        "ape": rnd(r, 2 * D), "iape": rnd(r, 2 * Di), "gamma": 1 + rnd(D, scale=0.02), "igamma": 1 + rnd(Di, scale=0.02),
        "score": rnd(B, T), "idx": torch.full((B, W + 64), 7, dtype=torch.int32, device=dev),
    }
    return s


@pytest.mark.parametrize("beside", [False, True])
@pytest.mark.parametrize("B", [64, 5])
def test_layer_prologue_equals_separate_calls(cuda_dev, B, beside):
    from dsv4attn import ops
    D, Di, W, T, r = 512, 128, 128, 1024, 4
    g = torch.Generator().manual_seed(B * 10 + int(beside))
    base = _state(B, D, Di, W, T, r, g, cuda_dev)
    a = {k: v.clone() for k, v in base.items()}
    b = {k: v.clone() for k, v in base.items()}
    cos, sin = (t.to(cuda_dev) for t in O.rope_tables(64, 8192, compressed=True))
    pos0 = torch.randint(400, 3000, (B,), generator=g, dtype=torch.int32)
    for step in range(6):
        pos = (pos0 + step).to(cuda_dev)
        ta = ((pos + 1) // r).to(torch.int32)
        tprev = (ta - 1).clamp_min(0)
        x = {"kv": torch.randn(B, D, generator=g).to(BF), "cmp_kv": torch.randn(B, 2 * D, generator=g).to(BF),
             "cmp_sc": torch.randn(B, 2 * D, generator=g).to(BF), "icmp_kv": torch.randn(B, 2 * Di, generator=g).to(BF),
             "icmp_sc": torch.randn(B, 2 * Di, generator=g).to(BF), "iq": torch.randn(B, 64, Di, generator=g).to(BF),
             "iw": 0.02 * torch.randn(B, 64, generator=g)}
        x = {k: v.to(cuda_dev) for k, v in x.items()}
        # separate calls
        ops.indexer_score(x["iq"], a["idx_cache"], x["iw"], T, out=a["score"], t_valid=tprev)
        ops.compressor_step(x["icmp_kv"], x["icmp_sc"], a["iape"], a["ikv_state"], a["isc_state"], a["igamma"], cos, sin,
                            a["idx_cache"], 0, pos, r, overlap=True, rotate=False, eps=1e-6, rope_dim=64)
        ops.indexer_score_newest(x["iq"], a["idx_cache"], x["iw"], ta, T, out=a["score"])
        ops.kv_window_write(x["kv"], a["kv_cache"], pos, W, rope_dim=64)
        ops.window_indices(pos, W, out=a["idx"][:, :W])
        ops.compressor_step(x["cmp_kv"], x["cmp_sc"], a["ape"], a["kv_state"], a["sc_state"], a["gamma"], cos, sin,
                            a["kv_cache"], W, pos, r, overlap=True, rotate=False, eps=1e-6, rope_dim=64)
        # one launch, after (beside) the score as in the decode step
        ops.indexer_score(x["iq"], b["idx_cache"], x["iw"], T, out=b["score"], t_valid=tprev)
        ops.layer_prologue((x["icmp_kv"], x["icmp_sc"], b["iape"], b["ikv_state"], b["isc_state"], b["igamma"],
                            b["idx_cache"]),
                           (x["cmp_kv"], x["cmp_sc"], b["ape"], b["kv_state"], b["sc_state"], b["gamma"], b["kv_cache"]),
                           cos, sin, pos, ta, x["iq"], x["iw"], b["score"], T, x["kv"], b["idx"], W, r, eps=1e-6,
                           rope_dim=64, beside_previous=beside)
        torch.cuda.synchronize()
        for k in base:
            assert torch.equal(a[k].cpu().view(torch.uint8), b[k].cpu().view(torch.uint8)) if a[k].dtype == BF \
                else torch.equal(a[k].cpu(), b[k].cpu()), f"step {step}: {k} differs"


def test_layer_prologue_rejects_bad_shapes(cuda_dev):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(1)
    B, D, Di, W, T, r = 2, 512, 128, 128, 256, 4
    s = _state(B, D, Di, W, T, r, g, cuda_dev)
    cos, sin = (t.to(cuda_dev) for t in O.rope_tables(64, 1024, compressed=True))
    pos = torch.full((B,), 10, dtype=torch.int32, device=cuda_dev)
    x = torch.zeros(B, 2 * Di, dtype=BF, device=cuda_dev)
    with pytest.raises(ValueError):   # the window row must be the attention compressor's width
        ops.layer_prologue((x, x, s["iape"], s["ikv_state"], s["isc_state"], s["igamma"], s["idx_cache"]),
                           (torch.zeros(B, 2 * D, dtype=BF, device=cuda_dev), torch.zeros(B, 2 * D, dtype=BF, device=cuda_dev),
                            s["ape"], s["kv_state"], s["sc_state"], s["gamma"], s["kv_cache"]),
                           cos, sin, pos, pos, torch.zeros(B, 64, Di, dtype=BF, device=cuda_dev),
                           torch.zeros(B, 64, device=cuda_dev), s["score"], T,
                           torch.zeros(B, 256, dtype=BF, device=cuda_dev), s["idx"], W, r)
