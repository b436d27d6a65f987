"""GPU parity straight against the reference's own chains.

The CUDA kernels run on the inputs stored in ``tests/golden/ref_chains.npz``
(produced by the reference's functions through the torch ttnn stand-in,
``tests/golden/make_ref_chains.py``) and are compared with the reference's
outputs directly, not only through the oracle:

* act_quant scales bit-exact with the chain's ``multiply(amax, 1/448)``;
* top-k index sets equal to ``_indexer_topk_body`` except at near-ties;
* sparse attention within rtol/atol 2e-2 (and relative error < 1e-2) of
  ``DeviceSparseAttn.forward_device``;
* indexer score within rtol 1e-3 of the Lk-D-idx-score reference;
* the compressor's emitted rows within rtol/atol 2e-2 of the ttnn compressor
  classes, its fp32 state equal to theirs.
"""

import os

import numpy as np
import pytest
import torch

import oracle as O
from parity import assert_topk_sets, masked_scores

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def chains():
    return np.load(os.path.join(HERE, "golden", "ref_chains.npz"))


def test_act_quant_scale_matches_chain(cuda_dev, chains):
    from dsv4attn import ops
    x = torch.from_numpy(chains["aq_x"]).to(torch.bfloat16)
    got, gs, _ = ops.act_quant_block(x.to(cuda_dev), scales=True)
    torch.cuda.synchronize()
    assert torch.equal(gs.cpu(), torch.from_numpy(chains["aq_scale"]))
    want, _, _ = O.act_quant_block(x)
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))


def test_topk_matches_chain(cuda_dev, chains):
    from dsv4attn import ops
    for ci in range(int(chains["tk_cases"])):
        score = torch.from_numpy(chains[f"tk{ci}_score"])[:, 0].contiguous()
        ta = torch.from_numpy(chains[f"tk{ci}_t_active"])
        bk, k, win = (int(v) for v in chains[f"tk{ci}_meta"])
        got = ops.indexer_topk(score.to(cuda_dev), ta.to(cuda_dev), k, win).cpu()
        want = torch.from_numpy(chains[f"tk{ci}_idx"])[:, 0]
        assert_topk_sets(got, want, masked_scores(score, ta), win, what=f"chain case {ci}")


def test_sparse_attn_matches_chain(cuda_dev, chains):
    from dsv4attn import ops
    q = torch.from_numpy(chains["sa_q"]).to(torch.bfloat16)            # [1, S, H, D], scale folded in
    kv = torch.from_numpy(chains["sa_kv"]).to(torch.bfloat16).unsqueeze(0)
    idx = torch.from_numpy(chains["sa_idx"])                             # [1, S, K]
    sink = torch.from_numpy(chains["sa_sink"])
    out = ops.sparse_attn(q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev), sink.to(cuda_dev), 1.0).cpu().float()
    want = torch.from_numpy(chains["sa_out"])
    torch.testing.assert_close(out, want, rtol=2e-2, atol=2e-2)
    live = want[0, :2]
    assert float((out[0, :2] - live).norm() / live.norm()) < 1e-2
    assert float(out[0, 2].abs().max()) == 0.0                          # sink-only row


def test_indexer_score_matches_chain(cuda_dev, chains):
    from dsv4attn import ops
    x = torch.from_numpy(chains["is_x"]).reshape(1, -1)
    w = ((x @ torch.from_numpy(chains["is_wproj"])) * float(chains["is_scale"])).contiguous()
    q = torch.from_numpy(chains["is_q"]).reshape(1, 64, 128).to(torch.bfloat16)
    k = torch.from_numpy(chains["is_kv"]).reshape(1, -1, 128).to(torch.bfloat16)
    T = k.shape[1]
    got = ops.indexer_score(q.to(cuda_dev), k.to(cuda_dev), w.to(cuda_dev), T).cpu()
    want = torch.from_numpy(chains["is_out"]).reshape(1, -1)
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3 * float(want.abs().max()))


@pytest.mark.parametrize("name,overlap", [("co", True), ("cn", False)])
def test_compressor_matches_chain(cuda_dev, chains, name, overlap):
    from dsv4attn import ops
    r = int(chains[f"{name}_ratio"])
    kv_in = torch.from_numpy(chains[f"{name}_kv_in"]).to(torch.bfloat16)
    sc_in = torch.from_numpy(chains[f"{name}_sc_in"]).to(torch.bfloat16)
    steps, B = kv_in.shape[0], kv_in.shape[1]
    dev = cuda_dev
    ape = torch.from_numpy(chains[f"{name}_ape"]).to(dev)
    gamma = torch.from_numpy(chains[f"{name}_gamma"]).to(dev)
    cos = torch.from_numpy(chains[f"{name}_cos"]).contiguous().to(dev)
    sin = torch.from_numpy(chains[f"{name}_sin"]).contiguous().to(dev)
    kv_s, sc_s = (t.to(dev) for t in O.compressor_init_state(B, 512, r, overlap))
    rows = chains[f"{name}_cache"].shape[1]
    cache = torch.zeros(B, rows, 512, dtype=torch.bfloat16, device=dev)
    emitted = torch.zeros(B, dtype=torch.int32, device=dev)
    for pos in range(steps):
        p = torch.full((B,), pos, dtype=torch.int32, device=dev)
        ops.compressor_step(kv_in[pos, :, 0].to(dev), sc_in[pos, :, 0].to(dev), ape, kv_s, sc_s, gamma, cos, sin,
                            cache, 0, p, r, overlap, emitted=emitted)
        assert bool(emitted.cpu().eq(1).all()) == bool(chains[f"{name}_emitted"][pos])
        if chains[f"{name}_emitted"][pos]:
            want = torch.from_numpy(chains[f"{name}_emits"][pos])
            torch.testing.assert_close(cache[:, pos // r].cpu().float(), want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kv_s.cpu(), torch.from_numpy(chains[f"{name}_kv_state"]), rtol=0, atol=0)
    torch.testing.assert_close(sc_s.cpu(), torch.from_numpy(chains[f"{name}_sc_state"]), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(cache.cpu().float(), torch.from_numpy(chains[f"{name}_cache"]), rtol=2e-2, atol=2e-2)
