"""Host-side checks of the reference-signature drop-ins that need no GPU:
the refusal of a CPU device (no CPU fallback), weight conversion, and the
block oracle the GPU parity tests rely on."""

import math

import pytest
import torch

import oracle.path as ref
from standins import make_block


def test_device_modules_refuse_cpu():
    from dsv4attn import modules as M
    with pytest.raises(ValueError, match="CUDA"):
        M.DeviceSparseAttn("cpu", torch.zeros(64), 0.1)
    with pytest.raises(ValueError, match="CUDA"):
        M.DeviceLinear(torch.device("cpu"), torch.zeros(4, 4))


def test_weight_bf16_expands_fp8_block_scales():
    from dsv4attn.modules import weight_bf16
    g = torch.Generator().manual_seed(0)
    w = torch.randn(200, 300, generator=g).to(torch.float8_e4m3fn)
    scale = torch.tensor([[2.0 ** i for i in range(3)], [2.0 ** -i for i in range(3)]])
    lin = type("L", (), {})()
    lin.weight = w
    lin.scale = scale
    got = weight_bf16(lin)
    exp = w.float().clone()
    for i in range(2):
        for j in range(3):
            exp[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128] *= scale[i, j]
    assert torch.equal(got, exp.to(torch.bfloat16))
    with pytest.raises(ValueError):
        weight_bf16(torch.zeros(2, 2, dtype=torch.int8))


def test_block_oracle_runs_and_matches_layer_step_pieces():
    """The block oracle equals its pieces chained by hand at one position."""
    B = 2
    attn, bw, st = make_block(seed=1, B=B, max_seq_len=256)
    x = torch.randn(B, 1, attn.dim, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    out = ref.attention_decode_block(bw, st, x, 3)
    assert out.shape == (B, 1, attn.dim) and out.dtype == torch.bfloat16
    assert torch.isfinite(out.float()).all()
    # the window row written at slot 3 is the Lk-D1 chain of wkv(x)
    kv = ref.linear_bf16(x.reshape(B, -1), bw.wkv)
    row, _, _ = ref.kv_norm_rope_quant(kv, bw.kv_norm, st.cos[3].expand(B, -1), st.sin[3].expand(B, -1))
    assert torch.equal(st.kv_cache[:, 3], row)
    # position 3 emits compressed row 0 into both caches
    assert st.kv_cache[:, st.win].abs().sum() > 0
    assert st.idx_kv_cache[:, 0].abs().sum() > 0


def test_head_norm_rope_oracle_identities():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 2 * 128, generator=g).to(torch.bfloat16)
    cos, sin = ref.rope_tables(64, 10, compressed=True)
    c, s = cos[[1, 5, 9]], sin[[1, 5, 9]]
    y = ref.head_norm_rope(x, 2, 128, c, s, 64, norm=False)
    back = ref.head_norm_rope(y, 2, 128, c, s, 64, norm=False, inverse=True)
    assert float((back.float() - x.float()).abs().max()) < 0.05
    assert torch.equal(y.view(3, 2, 128)[..., :64], x.view(3, 2, 128)[..., :64])
    n = ref.head_norm_rope(x, 2, 128, norm=True, weight=1.0)
    rms = n.float().view(3, 2, 128).pow(2).mean(-1).sqrt()
    assert torch.allclose(rms, torch.ones_like(rms), atol=2e-2)
