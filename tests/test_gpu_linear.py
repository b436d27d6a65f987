"""GPU parity of the decode projections' tcgen05 kernel (dsa_linear) with
the oracle's bf16 projection (fp32 accumulation, bf16 result;
inference.py:5934-5960): plain, ragged (N not a multiple of the 128-row
tile, B not a multiple of 16, B above one 128-row chunk), the head-grouped
wo_a form (inference.py:6105-6122), the fp32 copy of weights_proj
(5177-5185) and the q rotary fused into wq_b's epilogue (Lk-D-idx-q,
5226-5258), the latter bit-exact against the oracle's rotary applied to the
kernel's own un-rotated result."""

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _ref(x, w, G):
    """fp64 per-group projection (the accumulation-order-free value)."""
    B = x.shape[0]
    N, K = w.shape[0] // G, w.shape[1]
    xs = x.double().view(B, G, K)
    ws = w.double().view(G, N, K)
    return torch.einsum("bgk,gnk->bgn", xs, ws).reshape(B, G * N)


def _check(y, x, w, G):
    """bf16 result of an fp32-accumulated dot: within half a bf16 ulp of the
    exact value plus the fp32 accumulation error, |x|.|w| * K * 2^-23."""
    exact = _ref(x.cpu(), w.cpu(), G)
    K = w.shape[1]
    mag = torch.einsum("bgk,gnk->bgn", x.cpu().double().abs().view(x.shape[0], G, K),
                       w.cpu().double().abs().view(G, -1, K)).reshape(exact.shape)
    tol = exact.abs() * 2.0 ** -8 + mag * K * 2.0 ** -23 + 1e-30
    err = (y.cpu().double() - exact).abs()
    assert bool((err <= tol).all()), f"max err/tol {float((err / tol).max()):.3f}"
    # and the oracle's own bf16 projection agrees to one bf16 rounding (plus
    # both sides' fp32 accumulation error where the sum cancels)
    want = torch.cat([O.linear_bf16(x.cpu()[:, g * K:(g + 1) * K], w.cpu()[g * (w.shape[0] // G):
                                                                          (g + 1) * (w.shape[0] // G)])
                      for g in range(G)], 1)
    d = (y.cpu().double() - want.double()).abs()
    tol2 = want.double().abs() * 2.0 ** -7 + 2 * mag * K * 2.0 ** -23 + 1e-30
    assert bool((d <= tol2).all()), f"vs oracle: max err/tol {float((d / tol2).max()):.3f}"


@pytest.mark.parametrize("B,N,K,G", [(1, 384, 256, 1), (2, 200, 128, 1), (7, 128, 64, 1), (64, 512, 1024, 1),
                                     (130, 256, 192, 1), (3, 64, 256, 8), (5, 256, 128, 4), (64, 1024, 512, 8),
                                     (1, 64, 4096, 1), (4, 25600, 1024, 1), (16, 1024, 4096, 8), (128, 320, 2048, 1),
                                     (3, 100, 128, 2), (5, 36, 512, 3), (70, 96, 1024, 2), (40, 384, 64, 1),
                                     (72, 256, 64, 1), (128, 512, 4096, 1), (100, 2048, 8192, 1)])
def test_linear_matches_oracle(cuda_dev, B, N, K, G):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B * 1000 + N + K + G)
    x = torch.randn(B, G * K, generator=g).to(BF)
    w = (torch.randn(G * N, K, generator=g) * K ** -0.5).to(BF)
    y = ops.linear(x.to(cuda_dev), w.to(cuda_dev), groups=G)
    torch.cuda.synchronize()
    assert y.shape == (B, G * N) and y.dtype == BF
    _check(y, x, w, G)


def test_linear_strided_rows_and_out(cuda_dev):
    """x rows with a stride above G*K (a column slice of a wider buffer) and
    y written into a wider output buffer, columns past G*N untouched."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(5)
    big = torch.randn(9, 640, generator=g).to(BF)
    x = big[:, 64:64 + 256]
    w = (torch.randn(320, 256, generator=g) * 0.06).to(BF)
    out = torch.full((9, 400), 7.0, dtype=BF, device=cuda_dev)
    xd = big.to(cuda_dev)[:, 64:64 + 256]
    ops.linear(xd, w.to(cuda_dev), out=out)
    torch.cuda.synchronize()
    _check(out[:, :320], x.contiguous(), w, 1)
    assert bool((out[:, 320:].cpu() == 7.0).all())


@pytest.mark.parametrize("B,N,K", [(33, 64, 512), (64, 64, 4096), (3, 300, 128), (48, 256, 64), (128, 256, 4096)])
def test_linear_out_f32_is_the_bf16_value(cuda_dev, B, N, K):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(6)
    x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
    w = (torch.randn(N, K, generator=g) * 0.05).to(BF).to(cuda_dev)
    wp = ops.pack_linear_weight(w)
    yb = ops.linear(x, wp)
    yf = ops.linear(x, wp, out_f32=True)
    torch.cuda.synchronize()
    assert yf.dtype == torch.float32
    assert torch.equal(yf.cpu(), yb.cpu().float())


def test_linear_unaligned_output_rows(cuda_dev):
    """Y rows whose stride is not a multiple of 16 bytes (no TMA store):
    the element-wise stores give the same values."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(8)
    x = torch.randn(6, 256, generator=g).to(BF).to(cuda_dev)
    w = (torch.randn(128, 256, generator=g) * 0.06).to(BF).to(cuda_dev)
    wp = ops.pack_linear_weight(w)
    want = ops.linear(x, wp)
    out = torch.zeros(6, 131, dtype=BF, device=cuda_dev)
    ops.linear(x, wp, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out[:, :128].cpu(), want.cpu())
    assert bool((out[:, 128:].cpu() == 0).all())


@pytest.mark.parametrize("B,H,Dh,rd,K", [(5, 4, 128, 64, 128), (64, 64, 128, 64, 1024), (130, 2, 64, 32, 64),
                                         (40, 4, 128, 64, 64), (45, 8, 128, 64, 1024)])
def test_linear_fused_rotary_bit_exact(cuda_dev, B, H, Dh, rd, K):
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + H + Dh)
    max_seq = 4096
    cos, sin = O.rope_tables(rd, max_seq, compressed=True)
    pos = torch.randint(0, max_seq, (B,), generator=g, dtype=torch.int32)
    x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
    w = (torch.randn(H * Dh, K, generator=g) * K ** -0.5).to(BF).to(cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    plain = ops.linear(x, w)
    roped = ops.linear(x, w, rope=(cos.to(cuda_dev), sin.to(cuda_dev), pos.to(cuda_dev), Dh, rd), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = O.head_norm_rope(plain.cpu(), H, Dh, cos[pos.long()], sin[pos.long()], rope_dim=rd, norm=False)
    assert torch.equal(roped.cpu().view(torch.int16), want.view(torch.int16))


def test_linear_bad_position_sets_status(cuda_dev):
    from dsv4attn import ops
    cos, sin = O.rope_tables(64, 16, compressed=True)
    x = torch.ones(2, 64, dtype=BF, device=cuda_dev)
    w = torch.ones(128, 64, dtype=BF, device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    pos = torch.tensor([3, 99], dtype=torch.int32, device=cuda_dev)
    ops.linear(x, w, rope=(cos.to(cuda_dev), sin.to(cuda_dev), pos, 128, 64), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & ops.STATUS_BAD_INDEX


def test_linear_rejects_bad_shapes(cuda_dev):
    from dsv4attn import ops
    x = torch.ones(2, 96, dtype=BF, device=cuda_dev)
    with pytest.raises((ValueError, RuntimeError)):
        ops.linear(x, torch.ones(64, 96, dtype=BF, device=cuda_dev))    # K not a multiple of 64
    with pytest.raises(ValueError):
        ops.linear(torch.ones(2, 128, dtype=BF, device=cuda_dev), torch.ones(64, 64, dtype=BF, device=cuda_dev),
                   groups=3)


@pytest.mark.parametrize("B,N0,H,Dh,rd,K", [(64, 512, 4, 128, 64, 256), (3, 1024, 2, 128, 64, 128)])
def test_linear_rotary_from_column_bit_exact(cuda_dev, B, N0, H, Dh, rd, K):
    """Two projections of one input stored as one weight, the rotary on the
    second only (rope col0 = N0, the attention's wq_b next to the indexer's
    wq_b): columns before col0 untouched, the rest bit-exact against the
    oracle's rotary of the kernel's own unrotated result."""
    from dsv4attn import ops
    g = torch.Generator().manual_seed(B + N0)
    cos, sin = O.rope_tables(rd, 2048, compressed=True)
    pos = torch.randint(0, 2048, (B,), generator=g, dtype=torch.int32)
    x = torch.randn(B, K, generator=g).to(BF).to(cuda_dev)
    w = (torch.randn(N0 + H * Dh, K, generator=g) * K ** -0.5).to(BF).to(cuda_dev)
    wp = ops.pack_linear_weight(w)
    plain = ops.linear(x, wp)
    roped = ops.linear(x, wp, rope=(cos.to(cuda_dev), sin.to(cuda_dev), pos.to(cuda_dev), Dh, rd, N0))
    torch.cuda.synchronize()
    assert torch.equal(roped[:, :N0].cpu(), plain[:, :N0].cpu())
    want = O.head_norm_rope(plain[:, N0:].cpu(), H, Dh, cos[pos.long()], sin[pos.long()], rope_dim=rd, norm=False)
    assert torch.equal(roped[:, N0:].cpu().view(torch.int16), want.view(torch.int16))
