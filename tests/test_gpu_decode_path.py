"""GPU parity of the whole per-layer decode step (DecodePath) against the
oracle's decode_layer_step over many positions: window wrap-around, emits
of both compressors, indexer top-k and attention, eager and graph-replayed."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _make(cuda_dev, B=2, W=16, k=8, max_seq=160, seed=0):
    from dsv4attn.layer import DecodeLayer, DecodePath
    from dsv4attn.tables import PathArgs
    args = PathArgs(window_size=W, index_topk=k)
    L = DecodeLayer(args, B, max_seq, cuda_dev)
    g = torch.Generator().manual_seed(seed)
    L.ape.copy_(torch.randn(4, 1024, generator=g))
    L.gamma.copy_(1 + 0.02 * torch.randn(512, generator=g))
    L.iape.copy_(torch.randn(4, 256, generator=g))
    L.igamma.copy_(1 + 0.02 * torch.randn(128, generator=g))
    L.sink.copy_(torch.randn(64, generator=g))
    path = DecodePath([L], max_seq)
    cos, sin = O.rope_tables(64, max_seq, compressed=True)
    ckv, csc = O.compressor_init_state(B, 512, 4, True)
    ikv, isc = O.compressor_init_state(B, 128, 4, True)
    st = O.LayerState(kv_cache=torch.zeros(B, W + max_seq // 4, 512, dtype=torch.bfloat16),
                      idx_kv_cache=torch.zeros(B, max_seq // 4, 128, dtype=torch.bfloat16),
                      cmp_kv=ckv, cmp_sc=csc, icmp_kv=ikv, icmp_sc=isc, ape=L.ape.cpu(), gamma=L.gamma.cpu(),
                      iape=L.iape.cpu(), igamma=L.igamma.cpu(), sink=L.sink.cpu(), cos=cos, sin=sin,
                      win=W, ratio=4, index_topk=k, scale=512 ** -0.5)
    return path, L, st, g


def _inputs(g, B, dev):
    from dsv4attn.layer import LayerInputs
    bf = torch.bfloat16
    x = LayerInputs(q=torch.randn(B, 64, 512, generator=g).to(bf), kv=torch.randn(B, 512, generator=g).to(bf),
                    cmp_kv=torch.randn(B, 1024, generator=g).to(bf), cmp_score=torch.randn(B, 1024, generator=g).to(bf),
                    iq=torch.randn(B, 64, 128, generator=g).to(bf), icmp_kv=torch.randn(B, 256, generator=g).to(bf),
                    icmp_score=torch.randn(B, 256, generator=g).to(bf), iw=0.02 * torch.randn(B, 64, generator=g))
    xd = LayerInputs(*[t.to(dev) for t in x.tensors()])
    return x, xd


def _check_step(path, L, st, x, xd, pos, out):
    want_o, want_idx = O.decode_layer_step(st, pos, x.q.unsqueeze(1), x.kv, x.cmp_kv.float(), x.cmp_score.float(),
                                           x.iq, x.icmp_kv.float(), x.icmp_score.float(), x.iw)
    got_idx = L.idx.cpu()
    for b in range(got_idx.shape[0]):
        gs = set(int(v) for v in got_idx[b] if v >= 0)
        ws = set(int(v) for v in want_idx[b] if v >= 0)
        assert gs == ws, f"pos {pos} row {b}: index sets differ {sorted(gs ^ ws)}"
    torch.testing.assert_close(out.cpu().float(), want_o[:, 0].float(), rtol=2e-2, atol=2e-2)
    o, w = out.cpu().float(), want_o[:, 0].float()
    assert float((o - w).norm() / w.norm()) < 1e-2
    assert int(path.status.item()) == 0
    torch.testing.assert_close(L.kv_cache.cpu().float(), st.kv_cache.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(L.idx_cache.cpu().float(), st.idx_kv_cache.float(), rtol=2e-2, atol=2e-2)


def test_decode_path_eager_matches_oracle(cuda_dev):
    B = 2
    path, L, st, g = _make(cuda_dev, B=B)
    path.set_positions(0)
    out = torch.empty(B, 64, 512, dtype=torch.bfloat16, device=cuda_dev)
    for pos in range(0, 44):
        x, xd = _inputs(g, B, cuda_dev)
        path.step([xd], [out])
        torch.cuda.synchronize()
        assert int(path.pos[0]) == pos + 1
        _check_step(path, L, st, x, xd, pos, out)
    assert int(path.status.item()) == 0


def test_decode_path_graph_replay_matches_oracle(cuda_dev):
    from dsv4attn.layer import LayerInputs
    B = 2
    path, L, st, g = _make(cuda_dev, B=B, seed=1)
    out = torch.empty(B, 64, 512, dtype=torch.bfloat16, device=cuda_dev)
    xin = LayerInputs.empty(path.args, B, cuda_dev)
    for t in xin.tensors():
        t.zero_()
    # capture (warm-up steps advance state: re-create the layer state afterwards)
    path.capture([xin], [out], warmup=1)
    path2, L2, st2, g2 = _make(cuda_dev, B=B, seed=1)
    # copy the fresh state into the captured layer's buffers
    for a, b in [(L.kv_cache, L2.kv_cache), (L.idx_cache, L2.idx_cache), (L.cmp_kv, L2.cmp_kv),
                 (L.cmp_sc, L2.cmp_sc), (L.icmp_kv, L2.icmp_kv), (L.icmp_sc, L2.icmp_sc)]:
        a.copy_(b)
    path.set_positions(0)
    for pos in range(0, 24):
        x, xd = _inputs(g2, B, cuda_dev)
        xin.copy_(xd)
        path.replay()
        torch.cuda.synchronize()
        _check_step(path, L, st2, x, xd, pos, out)


def test_decode_path_config2_shapes_graph_matches_oracle(cuda_dev):
    """Config-2 shapes (window 128, top-2048 of 8192 compressed entries at a
    32k context) through the captured step the bench replays: side branches
    for the window write / attention compressor and the indexer compressor,
    the newest-row score recompute, programmatic dependent launches."""
    from dsv4attn.layer import DecodeLayer, DecodePath, LayerInputs
    from dsv4attn.tables import PathArgs
    from parity import assert_topk_sets, masked_scores
    B, W, k, ctx = 2, 128, 2048, 32768
    max_seq = ctx + 64
    pos0 = ctx - 3                      # steps cross an emit (pos % 4 == 3)
    args = PathArgs(window_size=W, index_topk=k)
    g = torch.Generator().manual_seed(77)
    T_max = max_seq // 4
    t0 = (pos0 + 1) // 4
    kv0 = torch.randn(B, W + T_max, 512, generator=g).to(torch.bfloat16)
    kv0[:, W + t0:] = 0
    keys0 = torch.randn(B, T_max, 128, generator=g).to(torch.bfloat16)
    keys0[:, t0:] = 0
    st_init = [torch.randn(B, 8, 1024, generator=g), torch.randn(B, 8, 1024, generator=g),
               torch.randn(B, 8, 256, generator=g), torch.randn(B, 8, 256, generator=g)]
    L = DecodeLayer(args, B, max_seq, cuda_dev)
    L.ape.copy_(torch.randn(4, 1024, generator=g))
    L.iape.copy_(torch.randn(4, 256, generator=g))
    L.sink.copy_(torch.randn(64, generator=g))
    path = DecodePath([L], max_seq)

    def load():
        L.kv_cache.copy_(kv0)
        L.idx_cache.copy_(keys0)
        for buf, v in zip((L.cmp_kv, L.cmp_sc, L.icmp_kv, L.icmp_sc), st_init):
            buf.copy_(v)
        path.set_positions(pos0)

    out = torch.empty(B, 64, 512, dtype=torch.bfloat16, device=cuda_dev)
    xin = LayerInputs.empty(args, B, cuda_dev)
    for t in xin.tensors():
        t.zero_()
    load()
    path.capture([xin], [out], warmup=1)
    load()
    cos, sin = O.rope_tables(64, max_seq, compressed=True)
    st = O.LayerState(kv_cache=kv0.clone(), idx_kv_cache=keys0.clone(), cmp_kv=st_init[0].clone(),
                      cmp_sc=st_init[1].clone(), icmp_kv=st_init[2].clone(), icmp_sc=st_init[3].clone(),
                      ape=L.ape.cpu(), gamma=L.gamma.cpu(), iape=L.iape.cpu(), igamma=L.igamma.cpu(),
                      sink=L.sink.cpu(), cos=cos, sin=sin, win=W, ratio=4, index_topk=k, scale=512 ** -0.5)
    for s in range(5):
        pos = pos0 + s
        x, xd = _inputs(g, B, cuda_dev)
        xin.copy_(xd)
        path.replay()
        torch.cuda.synchronize()
        want_o, want_idx = O.decode_layer_step(st, pos, x.q.unsqueeze(1), x.kv, x.cmp_kv.float(),
                                               x.cmp_score.float(), x.iq, x.icmp_kv.float(), x.icmp_score.float(),
                                               x.iw)
        got_idx = L.idx.cpu()
        assert torch.equal(got_idx[:, :W], want_idx[:, :W]), f"pos {pos}: window indices"
        t_active = (pos + 1) // 4
        assert_topk_sets(got_idx[:, W:], want_idx[:, W:], masked_scores(st.extra["score"], t_active), W,
                         what=f"pos {pos}")
        o, w = out.cpu().float(), want_o[:, 0].float()
        torch.testing.assert_close(o, w, rtol=2e-2, atol=2e-2)
        assert float((o - w).norm() / w.norm()) < 1e-2
        assert int(path.status.item()) == 0
    rows = W + (pos0 + 5) // 4 + 1
    torch.testing.assert_close(L.kv_cache[:, :rows].cpu().float(), st.kv_cache[:, :rows].float(), rtol=2e-2,
                               atol=2e-2)
    torch.testing.assert_close(L.idx_cache[:, :rows - W].cpu().float(), st.idx_kv_cache[:, :rows - W].float(),
                               rtol=2e-2, atol=2e-2)
