"""GPU parity: attn.kv (act_quant_block, window write) and attn.compress
(compressor state write / emit / slot shift) against the CPU oracle.

Bars: act_quant scales and e4m3 codes bit-exact, round-trip output
bit-exact; compressor rows within rtol 2e-2 / atol 2e-2 of the fp32 oracle
(in practice they agree to a bf16 ulp)."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def _edge_rows(n):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(n, 448, generator=g)
    x[0] = 0.0                                   # all-zero block -> eps floor
    x[1, :64] = 1e-7                              # tiny block
    x[2] = torch.randn(448, generator=g) * 1e4    # large magnitudes
    x[3, :64] = torch.tensor([448., -17., 19., 0.5] * 16)  # ties-to-even points
    x[4, 64:128] = -3.0                           # constant block
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("M", [1, 5, 32, 4096])
def test_act_quant_block_bit_exact(cuda_dev, M):
    from dsv4attn import ops
    x = _edge_rows(max(M, 5))[:M] if M >= 5 else torch.randn(M, 448).to(torch.bfloat16)
    want, ws, wq = O.act_quant_block(x)
    got, gs, gq = ops.act_quant_block(x.to(cuda_dev), scales=True, codes=True)
    torch.cuda.synchronize()
    assert torch.equal(gs.cpu(), ws), "scales differ"
    assert torch.equal(gq.cpu().view(torch.uint8), wq.view(torch.uint8)), "e4m3 codes differ"
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16)), "round-trip differs"


def test_act_quant_strided_rows(cuda_dev):
    from dsv4attn import ops
    base = torch.randn(8, 512).to(torch.bfloat16)
    x = base.to(cuda_dev)[:, :448]                 # row stride 512
    got, gs, _ = ops.act_quant_block(x, scales=True)
    want, ws, _ = O.act_quant_block(base[:, :448])
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))
    assert torch.equal(gs.cpu(), ws)


def test_kv_window_write(cuda_dev):
    from dsv4attn import ops
    B, D, W = 3, 512, 128
    kv = torch.randn(B, D).to(torch.bfloat16)
    pos = torch.tensor([0, 127, 4095], dtype=torch.int32)
    cache = torch.zeros(B, W + 16, D, dtype=torch.bfloat16)
    dc = cache.to(cuda_dev)
    scales = torch.zeros(B, 7, device=cuda_dev)
    ops.kv_window_write(kv.to(cuda_dev), dc, pos.to(cuda_dev), W, scales=scales)
    got = dc.cpu()
    for b in range(B):
        row, s, _ = O.kv_quant_row(kv[b:b + 1])
        slot = int(pos[b]) % W
        assert torch.equal(got[b, slot].view(torch.int16), row[0].view(torch.int16))
        assert torch.equal(scales[b].cpu(), s[0])
        other = torch.ones(W + 16, dtype=torch.bool)
        other[slot] = False
        assert (got[b][other] == 0).all()


def _run_compressor(cuda_dev, B, d, ratio, overlap, rotate, steps, slot_offset, start=0, seed=0):
    from dsv4attn import ops
    from dsv4attn.tables import PathArgs, rope_cos_sin
    g = torch.Generator().manual_seed(seed)
    coff = 2 if overlap else 1
    ape = torch.randn(ratio, coff * d, generator=g)
    gamma = 1 + 0.02 * torch.randn(d, generator=g)
    cos, sin = rope_cos_sin(PathArgs(), start + steps + 8, compressed=True)
    rows = slot_offset + (start + steps) // ratio + 2
    kv_s, sc_s = O.compressor_init_state(B, d, ratio, overlap)
    cache = torch.zeros(B, rows, d, dtype=torch.bfloat16)
    d_kv, d_sc, d_cache = kv_s.to(cuda_dev), sc_s.to(cuda_dev), cache.to(cuda_dev).clone()
    d_ape, d_gamma, d_cos, d_sin = ape.to(cuda_dev), gamma.to(cuda_dev), cos.to(cuda_dev), sin.to(cuda_dev)
    emitted = torch.zeros(B, dtype=torch.int32, device=cuda_dev)
    n_emit = 0
    for p in range(start, start + steps):
        kr = torch.randn(B, coff * d, generator=g).to(torch.bfloat16)
        sr = torch.randn(B, coff * d, generator=g).to(torch.bfloat16)
        want = O.compressor_step(kv_s, sc_s, kr, sr, ape, gamma, cos, sin, p, ratio, overlap, kv_cache=cache,
                                 slot_offset=slot_offset, rotate=rotate)
        pos = torch.full((B,), p, dtype=torch.int32, device=cuda_dev)
        ops.compressor_step(kr.to(cuda_dev), sr.to(cuda_dev), d_ape, d_kv, d_sc, d_gamma, d_cos, d_sin, d_cache,
                            slot_offset, pos, ratio, overlap, rotate=rotate, emitted=emitted)
        em = emitted.cpu()
        assert bool((em == 1).all()) == (want is not None) and bool((em == 0).all()) == (want is None)
        if want is not None:
            n_emit += 1
            got = d_cache[:, slot_offset + p // ratio].cpu().float()
            torch.testing.assert_close(got, want.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(d_kv.cpu(), kv_s, rtol=0, atol=0)
    torch.testing.assert_close(d_sc.cpu(), sc_s, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(d_cache.cpu().float(), cache.float(), rtol=2e-2, atol=2e-2)
    # rows agree to within one bf16 ulp almost everywhere
    diff = (d_cache.cpu().float() - cache.float()).abs()
    assert float((diff > 1e-2 * cache.float().abs().clamp_min(1e-3)).float().mean()) < 1e-3
    return n_emit


@pytest.mark.parametrize("d,rotate", [(512, False), (128, False), (128, True)])
def test_compressor_overlap_ratio4(cuda_dev, d, rotate):
    # attention compressor (d=512) and indexer compressor (d=128, rotate=True)
    n = _run_compressor(cuda_dev, B=3, d=d, ratio=4, overlap=True, rotate=rotate, steps=24, slot_offset=128)
    assert n == 6


def test_compressor_emit_at_pos3_slot7(cuda_dev):
    # start_pos 3 emits with state slot 7 (test_lk_d_comp.py:841-843)
    n = _run_compressor(cuda_dev, B=1, d=512, ratio=4, overlap=True, rotate=False, steps=4, slot_offset=0)
    assert n == 1


def test_compressor_non_overlap_cfg1(cuda_dev):
    # BASELINE config 1 form: batch 32, d 512, ratio 4, non-overlap, emit every 4th step
    n = _run_compressor(cuda_dev, B=32, d=512, ratio=4, overlap=False, rotate=False, steps=40, slot_offset=0)
    assert n == 10


def test_compressor_ratio128_non_overlap(cuda_dev):
    n = _run_compressor(cuda_dev, B=2, d=512, ratio=128, overlap=False, rotate=False, steps=256, slot_offset=128)
    assert n == 2


def test_compressor_emit_only_matches_fused(cuda_dev):
    """write_state=False is _emit_body alone (inference.py:4997): writing the
    last slot by hand and then emitting equals the fused step."""
    from dsv4attn import ops
    from dsv4attn.tables import PathArgs, rope_cos_sin
    B, d, r = 2, 512, 4
    g = torch.Generator().manual_seed(3)
    cos, sin = rope_cos_sin(PathArgs(), 64, compressed=True)
    cos, sin = cos.to(cuda_dev), sin.to(cuda_dev)
    ape = torch.randn(r, 2 * d, generator=g).to(cuda_dev)
    gamma = (1 + 0.02 * torch.randn(d, generator=g)).to(cuda_dev)
    st = []
    for _ in range(2):
        kv, sc = O.compressor_init_state(B, d, r, True)
        st.append([kv.to(cuda_dev), sc.to(cuda_dev), torch.zeros(B, 8, d, dtype=torch.bfloat16, device=cuda_dev)])
    for p in range(4):
        kr = torch.randn(B, 2 * d, generator=g).to(torch.bfloat16).to(cuda_dev)
        sr = torch.randn(B, 2 * d, generator=g).to(torch.bfloat16).to(cuda_dev)
        pos = torch.full((B,), p, dtype=torch.int32, device=cuda_dev)
        ops.compressor_step(kr, sr, ape, st[0][0], st[0][1], gamma, cos, sin, st[0][2], 0, pos, r, True)
        if p < 3:
            ops.compressor_step(kr, sr, ape, st[1][0], st[1][1], gamma, cos, sin, st[1][2], 0, pos, r, True)
        else:
            st[1][0][:, r + 3] = kr.float()
            st[1][1][:, r + 3] = sr.float() + ape[3]
            ops.compressor_step(None, None, None, st[1][0], st[1][1], gamma, cos, sin, st[1][2], 0, pos, r, True,
                                write_state=False)
    torch.cuda.synchronize()
    assert torch.equal(st[0][2], st[1][2])
    assert torch.equal(st[0][0], st[1][0]) and torch.equal(st[0][1], st[1][1])
