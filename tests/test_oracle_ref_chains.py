"""Pin the CPU oracle to outputs of the reference's OWN decode-path code.

``tests/golden/ref_chains.npz`` was produced by ``tests/golden/make_ref_chains.py``,
which runs the reference's functions (inference.py and its
device-compressor-indexer / tt-lang-kernels test modules) through a torch
stand-in for ttnn in fp32 arithmetic.  These tests check the oracle against
those outputs:

* act_quant (inference.py:4578-4607): output and scale bit-exact; the scale
  is ``multiply(amax, 1/448)``, which differs from ``amax / 448`` for about
  half of all inputs, so the choice is pinned, not incidental;
* the indexer top-k body (inference.py:5823-5851) and the verbatim Lk-D-topk
  reference chain (test_lk_d_topk.py:121-138): identical index rows, order
  included (both sort by value with torch.topk);
* sparse attention (inference.py:4444-4501): within 2e-6 of the chain;
* the indexer score reference (test_lk_d_idx_score.py:359-371): within 1e-7;
* the ttnn compressor classes (compressor_overlap.py, compressor_no_overlap.py):
  emitted rows bit-identical after the bf16 rounding, states identical.
"""

import os

import numpy as np
import pytest
import torch

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def chains():
    return np.load(os.path.join(HERE, "golden", "ref_chains.npz"))


def test_act_quant_matches_reference_chain(chains):
    x = torch.from_numpy(chains["aq_x"])
    out, s, _ = O.act_quant_fp32(x, e4m3=False)
    assert torch.equal(out.reshape(x.shape), torch.from_numpy(chains["aq_out"]))
    assert torch.equal(s.squeeze(-1), torch.from_numpy(chains["aq_scale"]))
    # the e4m3 round trip shares that scale and only rounds the codes
    xhat, s2, q = O.act_quant_block(x.to(torch.bfloat16))
    assert torch.equal(s2, torch.from_numpy(chains["aq_scale"]))
    assert torch.equal(q.float(), q.float().clamp(-448, 448))


def test_scale_choice_matters():
    # amax * fp32(1/448) and amax / 448 disagree for many amax values, so
    # following the chain's multiply is a real choice (inference.py:4602)
    a = torch.rand(64000, generator=torch.Generator().manual_seed(3)) * 500 + 1e-4
    mul = a * (1.0 / 448.0)
    div = a / 448.0
    assert int((mul != div).sum()) > 10000
    _, s, _ = O.act_quant_fp32(a.view(-1, 64), block=64, e4m3=False)
    amax = torch.maximum(a.view(-1, 64).abs().amax(-1, keepdim=True), torch.tensor(1e-4))
    assert torch.equal(s.view(-1, 1), amax * (1.0 / 448.0))
    assert not torch.equal(s.view(-1, 1), amax / 448.0)


def test_topk_body_matches_reference(chains):
    n = int(chains["tk_cases"])
    assert n >= 4
    for ci in range(n):
        score = torch.from_numpy(chains[f"tk{ci}_score"])[:, 0]
        ta = torch.from_numpy(chains[f"tk{ci}_t_active"])
        bk, k, win = (int(v) for v in chains[f"tk{ci}_meta"])
        got = O.indexer_topk(score, ta, k, win)
        want = torch.from_numpy(chains[f"tk{ci}_idx"])[:, 0]
        assert torch.equal(got, want), f"case {ci}"
        # rows whose T_active is below k end in -1 sentinels
        for b in range(score.shape[0]):
            assert int((want[b] < 0).sum()) == max(0, k - min(int(ta[b]), bk))


def test_topk_verbatim_reference_chain(chains):
    score = torch.from_numpy(chains["tkref_score"])[:, 0]
    bucket, k, win, t_active = (int(v) for v in chains["tkref_meta"])
    got = O.indexer_topk(score, t_active, k, win)
    assert torch.equal(got, torch.from_numpy(chains["tkref_idx"])[:, 0])


def test_sparse_attn_matches_reference(chains):
    q = torch.from_numpy(chains["sa_q"])[0]
    kv = torch.from_numpy(chains["sa_kv"])
    idx = torch.from_numpy(chains["sa_idx"])[0]
    sink = torch.from_numpy(chains["sa_sink"])
    m, l, o = O.sparse_attn_partial(q, kv.unsqueeze(0).expand(q.shape[0], -1, -1), idx, 1.0)
    got = O.lse_combine([(m, l, o)], sink.unsqueeze(0))
    want = torch.from_numpy(chains["sa_out"])[0]
    torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)
    # the reference's mask form: safe = clamp(idx, 0), valid = -inf where idx < 0
    assert torch.equal(torch.from_numpy(chains["sa_safe"]).view(idx.shape), idx.clamp_min(0).long())
    valid = torch.from_numpy(chains["sa_valid"]).view(idx.shape)
    assert torch.equal(torch.isinf(valid), idx < 0)
    # a row with nothing valid attends to the sink only: zero output
    assert float(want[2].abs().max()) == 0.0


def test_indexer_score_matches_reference(chains):
    x = torch.from_numpy(chains["is_x"]).reshape(1, -1)
    w = (x @ torch.from_numpy(chains["is_wproj"])) * float(chains["is_scale"])
    q = torch.from_numpy(chains["is_q"]).reshape(1, 64, 128)
    k = torch.from_numpy(chains["is_kv"]).reshape(1, -1, 128)
    got = O.indexer_score(q, k, w)
    torch.testing.assert_close(got, torch.from_numpy(chains["is_out"]).reshape(1, -1), rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("name,overlap", [("co", True), ("cn", False)])
def test_compressor_matches_reference_classes(chains, name, overlap):
    r = int(chains[f"{name}_ratio"])
    kv_in = torch.from_numpy(chains[f"{name}_kv_in"])
    sc_in = torch.from_numpy(chains[f"{name}_sc_in"])
    ape = torch.from_numpy(chains[f"{name}_ape"])
    gamma = torch.from_numpy(chains[f"{name}_gamma"])
    cos, sin = torch.from_numpy(chains[f"{name}_cos"]), torch.from_numpy(chains[f"{name}_sin"])
    steps, B = kv_in.shape[0], kv_in.shape[1]
    kv_s, sc_s = O.compressor_init_state(B, 512, r, overlap)
    emitted = chains[f"{name}_emitted"]
    n = 0
    for pos in range(steps):
        out = O.compressor_step(kv_s, sc_s, kv_in[pos, :, 0], sc_in[pos, :, 0], ape, gamma, cos, sin, pos, r,
                                overlap)
        assert (out is not None) == bool(emitted[pos])
        if out is not None:
            n += 1
            want = torch.from_numpy(chains[f"{name}_emits"][pos]).to(torch.bfloat16)
            assert torch.equal(out.view(torch.int16), want.view(torch.int16)), f"emit at pos {pos}"
    assert n == steps // r
    assert torch.equal(kv_s, torch.from_numpy(chains[f"{name}_kv_state"]))
    assert torch.equal(sc_s, torch.from_numpy(chains[f"{name}_sc_state"]))
