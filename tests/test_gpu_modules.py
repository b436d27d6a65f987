"""GPU parity of the reference-signature drop-ins (dsv4attn.modules) and the
row kernels around the path against the CPU oracle.

Bars: attention-path outputs within rtol 2e-2 / atol 2e-2 of the fp32
oracle; block outputs (which add the projections,
rounded to bf16 at each step on both sides) within a relative Frobenius
error of 2e-2; act_quant codes bit-exact where the pre-quant bf16 row is
the same."""

import math

import pytest
import torch

import oracle as O
import oracle.path as ref
from standins import make_block

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


def rel_err(got, want):
    g, w = got.float().cpu(), want.float().cpu()
    return float((g - w).norm() / w.norm().clamp_min(1e-30))


def _modules():
    from dsv4attn import modules as M
    return M


# ----------------------------------------------------------- row kernels

@pytest.mark.parametrize("H,Dh,rd,norm,gamma,inverse", [
    (64, 512, 64, True, False, False),    # q path: rms with weight softmax_scale + rotary
    (1, 1024, 0, True, True, False),      # q_norm over q_lora_rank
    (64, 128, 64, False, False, False),   # indexer q rotary only
    (64, 512, 64, False, False, True),    # inverse rotary on o
])
def test_head_norm_rope_matches_oracle(cuda_dev, H, Dh, rd, norm, gamma, inverse):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(H + Dh + rd)
    B = 5
    x = torch.randn(B, H * Dh, generator=g).to(BF16)
    cos, sin = ref.rope_tables(64, 4096, compressed=True)
    pos = torch.tensor([0, 1, 77, 4000, 4095], dtype=torch.int32)
    gm = (1 + 0.1 * torch.randn(Dh, generator=g)) if gamma else None
    w = 512 ** -0.5
    got = ops.head_norm_rope(x.to(cuda_dev), H, Dh, cos.to(cuda_dev), sin.to(cuda_dev), pos.to(cuda_dev),
                             rope_dim=rd, gamma=None if gm is None else gm.to(cuda_dev), weight=w, norm=norm,
                             inverse=inverse)
    want = ref.head_norm_rope(x, H, Dh, cos[pos.long()], sin[pos.long()], rd, gamma=gm, weight=w, norm=norm,
                              inverse=inverse)
    torch.cuda.synchronize()
    d = (got.float().cpu() - want.float()).abs()
    # one bf16 ulp of slack for the fp32 sum order of the norm
    assert float((d / want.float().abs().clamp_min(1e-3)).max()) < 1.6e-2
    assert float((got.float().cpu() == want.float()).float().mean()) > 0.97


def test_head_norm_rope_in_place_and_bad_position_flag(cuda_dev):
    from dsv4attn import ops
    B, H, Dh = 2, 4, 128
    x = torch.randn(B, H * Dh, device=cuda_dev).to(BF16)
    cos, sin = ref.rope_tables(64, 16, compressed=True)
    pos = torch.tensor([3, 99], dtype=torch.int32, device=cuda_dev)  # 99 is past the table
    st = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    y = ops.head_norm_rope(x, H, Dh, cos.to(cuda_dev), sin.to(cuda_dev), pos, rope_dim=64, norm=False, out=x,
                           status=st)
    assert y.data_ptr() == x.data_ptr()
    assert int(st.item()) == 1


def test_kv_norm_rope_window_write_matches_oracle(cuda_dev):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(21)
    B, D, W = 6, 512, 128
    kv = (3 * torch.randn(B, D, generator=g)).to(BF16)
    gamma = 1 + 0.05 * torch.randn(D, generator=g)
    cos, sin = ref.rope_tables(64, 8192, compressed=True)
    pos = torch.tensor([0, 5, 127, 128, 4095, 8191], dtype=torch.int32)
    cache = torch.zeros(B, W + 4, D, dtype=BF16, device=cuda_dev)
    out = torch.empty(B, D, dtype=BF16, device=cuda_dev)
    scales = torch.empty(B, 7, dtype=torch.float32, device=cuda_dev)
    ops.kv_norm_rope_window_write(kv.to(cuda_dev), gamma.to(cuda_dev), cos.to(cuda_dev), sin.to(cuda_dev),
                                  pos.to(cuda_dev), cache, W, kv_out=out, scales=scales)
    row, s_want, _ = ref.kv_norm_rope_quant(kv, gamma, cos[pos.long()], sin[pos.long()])
    torch.cuda.synchronize()
    got = out.cpu()
    # identical wherever the kernel's bf16 norm output agrees with the oracle's
    same = (got.float() == row.float()).float().mean()
    assert float(same) > 0.99
    assert rel_err(got, row) < 1e-2
    assert torch.allclose(scales.cpu(), s_want, rtol=1e-2)
    c = cache.cpu()
    for b in range(B):
        assert torch.equal(c[b, int(pos[b]) % W], got[b])


def test_fold_index_mask(cuda_dev):
    from dsv4attn import ops
    idx = torch.randint(-1, 1000, (3, 1, 77), dtype=torch.int32, device=cuda_dev)
    safe = idx.clamp_min(0)
    valid = torch.where(idx >= 0, torch.zeros((), device=cuda_dev), torch.tensor(float("-inf"), device=cuda_dev))
    got = ops.fold_index_mask(safe.contiguous(), valid.to(BF16).contiguous())
    assert torch.equal(got, idx)


# ------------------------------------------------------ DeviceSparseAttn

@pytest.mark.parametrize("B,S,N,K", [(1, 1, 4224, 640), (2, 2, 3000, 700)])
def test_device_sparse_attn_forward_host_drop_in(cuda_dev, B, S, N, K):
    M = _modules()
    g = torch.Generator().manual_seed(B * 100 + K)
    H, D = 64, 512
    q = torch.randn(B, S, H, D, generator=g).to(BF16)
    kv = torch.randn(B, N, D, generator=g).to(BF16)
    idx = torch.randint(-1, N, (B, S, K), generator=g, dtype=torch.int32)
    sink = torch.randn(H, generator=g)
    sa = M.DeviceSparseAttn(cuda_dev, sink, D ** -0.5)
    out = sa.forward(q, kv, idx)
    assert out.device.type == "cpu" and out.dtype == BF16 and out.shape == q.shape
    want = O.sparse_attn(q, kv, idx, sink, D ** -0.5)
    assert torch.allclose(out.float(), want.float(), rtol=2e-2, atol=2e-2)


def test_device_sparse_attn_forward_device_mask_pair_equals_sentinels(cuda_dev):
    M = _modules()
    g = torch.Generator().manual_seed(4)
    B, S, H, D, N, K = 1, 1, 64, 512, 5000, 640
    scale = D ** -0.5
    q = (torch.randn(B, S, H, D, generator=g) * scale).to(BF16)  # pre-scaled, as the reference's q
    kv = torch.randn(N, D, generator=g).to(BF16)
    idx = torch.randint(-1, N, (B, S, K), generator=g, dtype=torch.int32)
    sink = torch.randn(H, generator=g)
    sa = M.DeviceSparseAttn(cuda_dev, sink, scale)
    qd, kvd, idxd = q.to(cuda_dev), kv.to(cuda_dev), idx.to(cuda_dev)
    i1, v1 = sa._idxs_int_tile_to_idxs_and_mask(idxd, B, S, K)
    assert v1 is None and tuple(i1.shape) == (B, S * K)
    o1 = sa.forward_device(qd, kvd, i1, v1, S, K)
    safe = idxd.clamp_min(0).reshape(B, S * K)
    valid = torch.where(idxd >= 0, 0.0, float("-inf")).to(BF16).view(B, S, 1, K)
    o2 = sa.forward_device(qd, kvd, safe, valid, S, K)
    assert torch.equal(o1, o2)
    want = O.sparse_attn(q, kv.unsqueeze(0), idx, sink, 1.0)
    assert torch.allclose(o1.float().cpu(), want.float(), rtol=2e-2, atol=2e-2)
    with pytest.raises(ValueError):
        sa.forward_device(qd, kvd, i1, None, S, K + 1)


# ------------------------------------------------------ DeviceCompressor

@pytest.mark.parametrize("fused", [False, True])
def test_device_compressor_matches_oracle_over_steps(cuda_dev, fused):
    M = _modules()
    B = 2
    attn, bw, st = make_block(seed=5, B=B)
    comp = attn.compressor
    T = 64
    comp.kv_cache = torch.zeros(B, T, comp.head_dim)
    if fused:
        lin = M.DeviceLinear.fused(cuda_dev, [comp.wkv, comp.wgate])
        dc = M.DeviceCompressor(cuda_dev, comp, lin, lin, None)
    else:
        dc = M.DeviceCompressor(cuda_dev, comp, M.DeviceLinear(cuda_dev, comp.wkv),
                                M.DeviceLinear(cuda_dev, comp.wgate), None)
    with pytest.raises(RuntimeError):
        dc.forward_device(torch.zeros(B, attn.dim, device=cuda_dev, dtype=BF16), B, 0, torch.zeros(1))
    kv_s, sc_s = comp.kv_state[:B].clone(), comp.score_state[:B].clone()
    oc = torch.zeros(B, T, comp.head_dim, dtype=BF16)
    g = torch.Generator().manual_seed(9)
    for pos in range(13):
        x = torch.randn(B, attn.dim, generator=g).to(BF16)
        dc.pre_stage_decode(pos, B)
        with pytest.raises(ValueError):
            dc.forward_device(x.to(cuda_dev), B, pos, None)
        got = dc.forward_device(x.to(cuda_dev), B, pos, dc._pos_tt)
        want = ref.compressor_step(kv_s, sc_s, ref.linear_bf16(x, comp.wkv.weight),
                                   ref.linear_bf16(x, comp.wgate.weight), comp.ape, comp.norm.weight, st.cos,
                                   st.sin, pos, 4, True, kv_cache=oc, slot_offset=0)
        if want is None:
            assert got is None
        else:
            assert got is not None and tuple(got.shape) == (B, 1, comp.head_dim)
            assert torch.allclose(got.float().cpu().squeeze(1), want.float(), rtol=2e-2, atol=2e-2)
    torch.cuda.synchronize()
    assert torch.allclose(dc.kv_state.cpu(), kv_s, rtol=1e-2, atol=1e-2)
    fin = torch.isfinite(sc_s)
    assert torch.equal(torch.isfinite(dc.score_state.cpu()), fin)
    assert torch.allclose(dc.score_state.cpu()[fin], sc_s[fin], rtol=1e-2, atol=1e-2)
    assert torch.allclose(dc.kv_cache_tt.float().cpu(), oc.float(), rtol=2e-2, atol=2e-2)


# --------------------------------------------------------- DeviceIndexer

def test_device_indexer_score_matches_oracle(cuda_dev):
    M = _modules()
    B = 2
    attn, bw, st = make_block(seed=7, B=B)
    ind = attn.indexer
    ic = ind.compressor
    ic.kv_cache = ind.kv_cache
    idc = M.DeviceCompressor(cuda_dev, ic, M.DeviceLinear(cuda_dev, ic.wkv), M.DeviceLinear(cuda_dev, ic.wgate),
                             None)
    di = M.DeviceIndexer(cuda_dev, ind, idc)
    Hi, Di = ind.n_heads, ind.head_dim
    kv_s, sc_s = ic.kv_state[:B].clone(), ic.score_state[:B].clone()
    oc = torch.zeros(B, ind.kv_cache.shape[1], Di, dtype=BF16)
    g = torch.Generator().manual_seed(13)
    wscale = Di ** -0.5 * Hi ** -0.5
    for pos in range(12):
        x = torch.randn(B, attn.dim, generator=g).to(BF16)
        qr = torch.randn(B, attn.q_lora_rank, generator=g).to(BF16)
        idc.pre_stage_decode(pos, B)
        score = di.forward_device_score(x.to(cuda_dev), qr.to(cuda_dev), B, pos, idc._pos_tt)
        iq = ref.head_norm_rope(ref.linear_bf16(qr, ind.wq_b.weight), Hi, Di, st.cos[pos].expand(B, -1),
                                st.sin[pos].expand(B, -1), 64, norm=False).view(B, Hi, Di)
        ref.compressor_step(kv_s, sc_s, ref.linear_bf16(x, ic.wkv.weight), ref.linear_bf16(x, ic.wgate.weight),
                            ic.ape, ic.norm.weight, st.cos, st.sin, pos, 4, True, kv_cache=oc, slot_offset=0)
        iw = ref.linear_bf16(x, (ind.weights_proj.weight.float() * wscale).to(BF16)).float()
        want = ref.indexer_score(iq, oc, iw)
        assert tuple(score.shape) == (B, 1, oc.shape[1])
        t_act = (pos + 1) // 4
        if t_act:
            assert rel_err(score[:, 0, :t_act], want[:, :t_act]) < 2e-2


# -------------------------------------------------------- DeviceAttention

def _block_run(cuda_dev, attn, bw, st, positions, B, seed, merged=True):
    M = _modules()
    if not merged:
        # twins bound beforehand (as the reference's offload binds them): the
        # block then runs every projection separately
        comp, ind = attn.compressor, attn.indexer
        attn._device_compressor = M.DeviceCompressor(cuda_dev, comp, M.DeviceLinear(cuda_dev, comp.wkv),
                                                     M.DeviceLinear(cuda_dev, comp.wgate), None)
        ic = ind.compressor
        attn._device_indexer = M.DeviceIndexer(cuda_dev, ind, M.DeviceCompressor(
            cuda_dev, ic, M.DeviceLinear(cuda_dev, ic.wkv), M.DeviceLinear(cuda_dev, ic.wgate), None))
    da = M.DeviceAttention(cuda_dev, attn, max_seq_len=st.cos.shape[0])
    assert (da._merged is not None) == merged
    g = torch.Generator().manual_seed(seed)
    for pos in positions:
        x = torch.randn(B, 1, attn.dim, generator=g).to(BF16)
        got = da.forward(x, pos)
        want = ref.attention_decode_block(bw, st, x, pos)
        assert got.shape == (B, 1, attn.dim) and got.dtype == BF16
        e = rel_err(got, want)
        assert e < 2e-2, f"pos {pos}: relative error {e}"
    assert int(da.status.item()) == 0
    return da


def test_device_attention_block_first_steps(cuda_dev):
    B = 2
    attn, bw, st = make_block(seed=11, B=B)
    _block_run(cuda_dev, attn, bw, st, range(0, 10), B, 1)


def test_device_attention_block_separate_projections(cuda_dev):
    """The same block with its compressor / indexer twins bound beforehand:
    nine separate projection launches instead of the merged ones."""
    B = 2
    attn, bw, st = make_block(seed=11, B=B)
    _block_run(cuda_dev, attn, bw, st, range(0, 6), B, 1, merged=False)


def test_device_attention_block_prefilled_selection(cuda_dev):
    """Resume at position 701 with filled caches and states, index_topk 64
    < T_active 175, so the indexer really selects; crosses the emit at 703."""
    B = 2
    attn, bw, st = make_block(seed=17, B=B, index_topk=64, max_seq_len=1024)
    g = torch.Generator().manual_seed(99)
    kv = torch.randn(attn.kv_cache.shape, generator=g).to(BF16)
    attn.kv_cache.copy_(kv.float())
    st.kv_cache.copy_(kv)
    ik = torch.randn(attn.indexer.kv_cache.shape, generator=g).to(BF16)
    attn.indexer.kv_cache.copy_(ik.float())
    st.idx_kv_cache.copy_(ik)
    for comp, okv, osc in ((attn.compressor, st.cmp_kv, st.cmp_sc), (attn.indexer.compressor, st.icmp_kv,
                                                                    st.icmp_sc)):
        comp.kv_state.copy_(torch.randn(comp.kv_state.shape, generator=g).to(BF16).float())
        comp.score_state.copy_(torch.randn(comp.score_state.shape, generator=g).to(BF16).float())
        okv.copy_(comp.kv_state)
        osc.copy_(comp.score_state)
    _block_run(cuda_dev, attn, bw, st, range(701, 706), B, 2)


def test_indexer_topk_body_reference_semantics(cuda_dev):
    M = _modules()
    B = 1
    attn, bw, st = make_block(seed=3, B=B)
    da = M.DeviceAttention(cuda_dev, attn, max_seq_len=1024)
    da.pre_stage_decode(199, B=B)  # T_active = 50
    g = torch.Generator().manual_seed(5)
    score = torch.randn(B, 1, 256, generator=g)
    da._indexer_score_in_tt = score.to(cuda_dev)
    out = da._indexer_topk_body(128, 64, 128, B, 1)
    want = O.indexer_topk(score[:, 0, :128], 50, 64, 128)
    assert tuple(out.shape) == (B, 1, 64)
    assert torch.equal(out.cpu().view(B, 64), want)
    with pytest.raises(RuntimeError):
        da.pre_stage_decode(5, B=B, S=2)
