"""Pin the CPU oracle against the reference's own helpers (golden fixtures
made by tests/golden/make_golden.py) and against known answers taken from
the reference's docstrings and ttnn op chains."""

import math

import numpy as np
import pytest
import torch

import oracle as O


# ----------------------------------------------------------------- golden pins

@pytest.mark.parametrize("win", [4, 8, 128])
def test_window_table_matches_reference(golden, win):
    np.testing.assert_array_equal(O.window_table(win).numpy(), golden[f"window_table_{win}"])


def test_window_row_pick_matches_reference(golden):
    table = golden["window_table_128"]
    for p, row in zip(golden["window_row_pos"], golden["window_row_128"]):
        np.testing.assert_array_equal(O.window_indices(int(p), 128).numpy(), table[row])


def test_shift_matches_reference_matrix(golden):
    state = torch.from_numpy(golden["shift_in"]).unsqueeze(0)          # [1, 32, 16]
    got = O.shift_matrix_apply(state, 4)[0].numpy()
    np.testing.assert_allclose(got, golden["shift_out"], rtol=0, atol=0)


def test_cssn_masks_define_overlap_view(golden):
    # mask_front rows [0,r), mask_back rows [r,2r), pad rows >= 2r
    mf, mb, mp = golden["cssn_mf"], golden["cssn_mb"], golden["cssn_mp"]
    assert (mf[:4] == 1).all() and (mf[4:] == 0).all()
    assert (mb[4:8] == 1).all() and (mb[:4] == 0).all() and (mb[8:] == 0).all()
    assert (mp[8:] == 1).all() and (mp[:8] == 0).all()


@pytest.mark.parametrize("kind", ["cmp", "dense"])
def test_yarn_tables_match_reference(golden, kind):
    rows = golden["freqs_rows"]
    cos, sin = O.rope_tables(64, int(rows.max()) + 1, compressed=(kind == "cmp"))
    np.testing.assert_allclose(cos[rows].numpy(), golden[f"freqs_{kind}_cos"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(sin[rows].numpy(), golden[f"freqs_{kind}_sin"], rtol=0, atol=2e-6)


def test_rotary_convention_matches_reference(golden):
    rows = golden["rot_rows"]
    cos, sin = O.rope_tables(64, int(rows.max()) + 1, compressed=True)
    x = torch.from_numpy(golden["rot_x"])
    got = O.rotary_interleaved(x, cos[rows], sin[rows])
    np.testing.assert_allclose(got.numpy(), golden["rot_out"], rtol=1e-5, atol=2e-5)
    inv = O.rotary_interleaved(x, cos[rows], sin[rows], inverse=True)
    np.testing.assert_allclose(inv.numpy(), golden["rot_inv_out"], rtol=1e-5, atol=2e-5)


def test_hadamard_matches_reference(golden):
    got = O.hadamard_rotate(torch.from_numpy(golden["had_x"]))
    np.testing.assert_allclose(got.numpy(), golden["had_out"], rtol=1e-5, atol=1e-5)


def test_compressor_state_init_matches_reference(golden):
    kv, sc = O.compressor_init_state(2, 512, 4, overlap=True)
    np.testing.assert_array_equal(kv.numpy(), golden["cmp_kv_state"])
    np.testing.assert_array_equal(sc.numpy(), golden["cmp_score_state"])
    kv128, _ = O.compressor_init_state(2, 512, 128, overlap=False)
    assert tuple(kv128.shape) == tuple(golden["cmp128_state_shape"])


def test_reference_constants(golden):
    assert tuple(golden["attn_kv_cache_shape"]) == (2, 128 + 64 // 4, 512)
    assert math.isclose(float(golden["attn_softmax_scale"]), 512 ** -0.5)
    assert int(golden["index_topk"]) == 512


# ------------------------------------------------------------ known answers

def test_act_quant_grid_values_are_identity():
    # a block whose max is 448 * 2^-3 holds values exactly on the e4m3 grid
    # scaled by s = 2^-3: the round trip must return them unchanged.
    s = 2.0 ** -3
    codes = torch.tensor([448., -448., 1., -0.5, 0.015625, 0., 240., -3.5] * 8)
    x = (codes * s).to(torch.bfloat16).unsqueeze(0)
    xhat, scales, q = O.act_quant_block(x)
    assert float(scales[0, 0]) == s
    torch.testing.assert_close(xhat.float(), x.float(), rtol=0, atol=0)
    torch.testing.assert_close(q.float(), codes.unsqueeze(0), rtol=0, atol=0)


def test_act_quant_eps_floor_and_rounding():
    x = torch.zeros(1, 128, dtype=torch.bfloat16)
    x[0, 64:] = 1e-6
    xhat, s, q = O.act_quant_block(x)
    assert float(s[0, 0]) == np.float32(1e-4) / np.float32(448.0)
    assert float(s[0, 1]) == float(s[0, 0])          # amax 1e-6 < eps floor
    assert (xhat[0, :64] == 0).all()
    # 17 lies between e4m3 grid points 16 and 18 -> ties-to-even gives 16
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    x[0, 0] = 448.0
    x[0, 1] = 17.0
    x[0, 2] = 19.0
    _, s, q = O.act_quant_block(x)
    assert float(s[0, 0]) == 1.0
    assert [float(v) for v in q[0, :3].float()] == [448.0, 16.0, 20.0]


def test_topk_one_hot_and_mask():
    # T_PAD 128, k 64, T_active 50 as in test_lk_d_topk.py:42-46, 219-224
    score = torch.full((1, 128), -5.0)
    score[0, 7] = 3.0
    score[0, 60] = 9.0          # beyond T_active: masked by -1e4, invalid
    idx = O.indexer_topk(score, 50, 64, win=128)
    assert idx.shape == (1, 64)
    assert int(idx[0, 0]) == 7 + 128
    valid = idx[0][idx[0] >= 0]
    assert valid.numel() == 50 and set(valid.tolist()) == set(range(128, 178))
    assert (idx[0, 50:] == -1).all()


def test_compressor_equal_gates_give_mean():
    # equal scores -> uniform softmax -> mean of the viewed rows, then RMSNorm
    B, d, r = 1, 8, 4
    kv, sc = O.compressor_init_state(B, d, r, overlap=False)
    rows = torch.arange(r * d, dtype=torch.float32).reshape(r, d)
    kv[0] = rows
    sc[0] = 0.0
    gamma = torch.ones(d)
    cos = torch.ones(1, 2)
    sin = torch.zeros(1, 2)
    out = O.compressor_emit(kv, sc, gamma, cos[0], sin[0], r, overlap=False, rope_dim=4)
    mean = rows.mean(0)
    want = mean * torch.rsqrt(mean.square().mean() + 1e-6)
    torch.testing.assert_close(out[0].float(), want.to(torch.bfloat16).float())


def test_compressor_overlap_view_uses_front_and_back_halves():
    B, d, r = 1, 4, 4
    kv, sc = O.compressor_init_state(B, d, r, overlap=True)
    kv[0, :r, :d] = 1.0         # front half of previous block
    kv[0, r:, d:] = 3.0         # back half of current block
    kv[0, :r, d:] = 100.0       # must be ignored by the view
    kv[0, r:, :d] = -100.0
    sc[0] = 0.0
    out = O.compressor_emit(kv, sc, torch.ones(d), torch.ones(1), torch.zeros(1), r,
                            overlap=True, rope_dim=2)
    assert torch.allclose(out.float(), torch.ones(1, d), atol=1e-2)  # mean 2 -> normed 1


def test_compressor_step_emits_and_shifts():
    B, d, r = 2, 16, 4
    torch.manual_seed(0)
    kv, sc = O.compressor_init_state(B, d, r, overlap=True)
    ape = torch.randn(r, 2 * d)
    cos, sin = O.rope_tables(4, 16, compressed=True)
    cache = torch.zeros(B, 8, d, dtype=torch.bfloat16)
    outs = []
    for pos in range(8):
        o = O.compressor_step(kv, sc, torch.randn(B, 2 * d), torch.randn(B, 2 * d), ape,
                              torch.ones(d), cos, sin, pos, r, True, kv_cache=cache,
                              slot_offset=2, rope_dim=4)
        outs.append(o)
    assert [o is not None for o in outs] == [False, False, False, True] * 2
    torch.testing.assert_close(cache[:, 2], outs[3])
    torch.testing.assert_close(cache[:, 3], outs[7])
    # after an emit, front rows equal back rows
    torch.testing.assert_close(kv[:, :r], kv[:, r:])


def test_sparse_attn_single_valid_index_and_sink():
    H, D, N = 4, 8, 6
    torch.manual_seed(1)
    q = torch.randn(1, 1, H, D).to(torch.bfloat16)
    kv = torch.randn(1, N, D).to(torch.bfloat16)
    idx = torch.tensor([[[-1, 3, -1]]], dtype=torch.int32)
    sink = torch.randn(H)
    o = O.sparse_attn(q, kv, idx, sink, 0.5)
    z = (q[0, 0].float() @ kv[0, 3].float()) * 0.5
    m = torch.maximum(z, sink)
    p = torch.exp(z - m) / (torch.exp(z - m) + torch.exp(sink - m))
    want = p.unsqueeze(-1) * kv[0, 3].float()
    torch.testing.assert_close(o[0, 0].float(), want, rtol=1e-2, atol=1e-2)


def test_sparse_attn_all_masked_gives_zero():
    q = torch.randn(1, 1, 2, 8).to(torch.bfloat16)
    kv = torch.randn(1, 4, 8).to(torch.bfloat16)
    idx = torch.full((1, 1, 3), -1, dtype=torch.int32)
    o = O.sparse_attn(q, kv, idx, torch.zeros(2), 1.0)
    assert (o == 0).all()


def test_lse_combine_equals_unsplit():
    torch.manual_seed(2)
    M, H, D, N, K = 2, 4, 16, 40, 24
    q = torch.randn(M, H, D).to(torch.bfloat16)
    kv = torch.randn(M, N, D).to(torch.bfloat16)
    idx = torch.randint(-1, N, (M, K), dtype=torch.int32)
    sink = torch.randn(H)
    full = O.sparse_attn(q, kv, idx, sink, 0.25).float()
    parts = [O.sparse_attn_partial(q, kv, idx[:, s:s + 8], 0.25) for s in range(0, K, 8)]
    comb = O.lse_combine(parts, sink.unsqueeze(0))
    torch.testing.assert_close(comb, full, rtol=1e-2, atol=1e-2)


def test_topk_merge_matches_global():
    torch.manual_seed(3)
    score = torch.randn(1, 4096)
    want = O.indexer_topk(score, 4096, 256, win=0)[0]
    cands_s, cands_i = [], []
    for g in range(4):
        sub = score[:, g * 1024:(g + 1) * 1024]
        v, i = torch.topk(sub, 256)
        cands_s.append(v[0])
        cands_i.append(i[0] + g * 1024)
    s, i = O.topk_merge(torch.cat(cands_s), torch.cat(cands_i), 256)
    assert set(i.tolist()) == set(want.tolist())


def test_decode_layer_step_runs():
    torch.manual_seed(4)
    B, H, D, Hi, Di, W, r = 2, 4, 512, 4, 128, 8, 4
    Tmax = 16
    cos, sin = O.rope_tables(64, 64, compressed=True)
    ckv, csc = O.compressor_init_state(B, D, r, True)
    ikv, isc = O.compressor_init_state(B, Di, r, True)
    st = O.LayerState(kv_cache=torch.zeros(B, W + Tmax, D, dtype=torch.bfloat16),
                      idx_kv_cache=torch.zeros(B, Tmax, Di, dtype=torch.bfloat16),
                      cmp_kv=ckv, cmp_sc=csc, icmp_kv=ikv, icmp_sc=isc,
                      ape=torch.randn(r, 2 * D), gamma=torch.ones(D),
                      iape=torch.randn(r, 2 * Di), igamma=torch.ones(Di),
                      sink=torch.randn(H), cos=cos, sin=sin, win=W, ratio=r, index_topk=3)
    for pos in range(12):
        o, idx = O.decode_layer_step(
            st, pos, torch.randn(B, 1, H, D).to(torch.bfloat16), torch.randn(B, D).to(torch.bfloat16),
            torch.randn(B, 2 * D), torch.randn(B, 2 * D), torch.randn(B, Hi, Di).to(torch.bfloat16),
            torch.randn(B, 2 * Di), torch.randn(B, 2 * Di), torch.randn(B, Hi) * 0.02)
        assert torch.isfinite(o.float()).all()
    assert idx.shape[-1] == W + 3
