"""The allocation-free attention entry point (dsa_sparse_attn_noalloc).

It exists for callers that cannot allocate device memory where they call
the attention; it keeps its split-K scratch in a fixed 8 MiB device array
instead of a caller workspace.  These tests call it through the C ABI and
check it against dsa_sparse_attn (the entry point that takes a workspace)
on two calls in a row, so stale scratch from the first call would show up
in the second.  This file is collected last on purpose."""

import pytest
import torch

from dsv4attn import _lib, ops

pytestmark = pytest.mark.gpu

ATTN_REL = 1e-2  # the relative error bound the attention parity tests use


def _case(B, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, 1, 64, 512, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, N, 512, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, N, (B, 1, K), generator=g, dtype=torch.int32)
    idx[torch.rand(B, 1, K, generator=g) < 0.1] = -1
    sink = torch.randn(64, generator=g)
    return q, kv, idx, sink


def _noalloc(q, kv, idx, sink, scale, status):
    B, S, H, D = q.shape
    K = idx.shape[-1]
    out = torch.empty_like(q)
    lse = torch.empty(B * S, H, device=q.device)
    rc = _lib.lib().dsa_sparse_attn_noalloc(
        q.data_ptr(), kv.data_ptr(), kv.stride(0), kv.shape[1], idx.data_ptr(), idx.stride(-2),
        sink.data_ptr(), out.data_ptr(), lse.data_ptr(), B, S, H, D, K, scale, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "sparse_attn_noalloc")
    return out, lse


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


@pytest.mark.parametrize("B,N,K", [(1, 70000, 2176), (2, 3000, 1000)])
def test_noalloc_matches_workspace_entry_point_twice(cuda_dev, B, N, K):
    scale = 512 ** -0.5
    lib = _lib.lib()
    assert lib.dsa_sparse_attn_workspace_size(B, 1, 64, 512, K) > 0, "shape must exercise the scratch"
    for call in range(2):
        q, kv, idx, sink = (t.to(cuda_dev) for t in _case(B, N, K, seed=100 * call + B))
        status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
        got, got_lse = _noalloc(q, kv, idx, sink, scale, status)
        want_lse = torch.empty(B, 64, device=cuda_dev)
        want = ops.sparse_attn(q, kv, idx, sink, scale, lse=want_lse)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
        assert _rel(got, want) < ATTN_REL
        torch.testing.assert_close(got_lse, want_lse, rtol=1e-3, atol=1e-3)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_dev):
    B, K = 64, 2176
    need = _lib.lib().dsa_sparse_attn_workspace_size(B, 1, 64, 512, K)
    assert need > 8 << 20
    q, kv, idx, sink = (t.to(cuda_dev) for t in _case(B, 300, K, seed=7))
    with pytest.raises(ValueError, match="maximum"):
        _noalloc(q, kv, idx, sink, 0.05, torch.zeros(1, dtype=torch.int32, device=cuda_dev))
