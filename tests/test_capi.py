"""C-ABI library checks that need no GPU: it loads, exports every entry point
declared in include/dsv4attn.h, the ctypes prototypes agree with the
header, and argument validation fails on the host with the reference's
Python error types (ValueError for shapes, inference.py:3036-3044)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "dsv4attn.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dsa_[a-z0-9_]+)\s*\(", src)))


def header_arg_counts():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(dsa_[a-z0-9_]+)\s*\(([^;]*?)\)\s*;", src, flags=re.S):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


def test_library_builds_and_loads():
    from dsv4attn import _lib
    L = _lib.lib()
    assert L.dsa_version() >= 100


def test_every_header_symbol_is_exported():
    from dsv4attn import _lib
    so = ctypes.CDLL(_lib.LIB_PATH)
    names = header_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(so, n), f"{n} declared in dsv4attn.h but not exported"


def test_prototypes_match_header():
    from dsv4attn import _lib
    counts = header_arg_counts()
    assert set(counts) == set(_lib.PROTOTYPES), set(counts) ^ set(_lib.PROTOTYPES)
    for name, (_, args) in _lib.PROTOTYPES.items():
        assert len(args) == counts[name], f"{name}: ctypes {len(args)} args, header {counts[name]}"


def test_host_validation_rejects_bad_shapes_without_launch():
    from dsv4attn import _lib
    L = _lib.lib()
    # indexer built for H=64, Di=128 only: rejected before any CUDA call
    rc = L.dsa_indexer_score(1, 1, 1, 1, None, 1, 32, 128, 16, 16 * 128, 16, None)
    assert rc == _lib.DSA_ERR_ARG
    assert "H=64" in _lib.last_error()
    with pytest.raises(ValueError, match="indexer_score"):
        _lib.check(rc, "indexer_score")
    # act_quant: N not divisible by block (ttnn chain's ValueError, inference.py:4597-4598)
    rc = L.dsa_act_quant_block(1, 1, None, None, 1, 100, 100, 100, 64, 448.0, 1e-4, None)
    assert rc == _lib.DSA_ERR_ARG and "divisible" in _lib.last_error()
    # top-k with k > T
    rc = L.dsa_indexer_topk(1, 8, 1, 1, None, 16, 1, 8, 16, 128, 0, 0, None)
    assert rc == _lib.DSA_ERR_ARG
    # sparse attention only built for H=64, D=512
    rc = L.dsa_sparse_attn(1, 1, 512, 1, 1, 4, 1, 1, None, 1, 1, 8, 512, 4, 1.0, None, 0, None, None)
    assert rc == _lib.DSA_ERR_ARG
    # null pointers
    assert L.dsa_kv_window_write(None, None, None, None, 1, 512, 64, 512 * 128, 128, 64, None) == _lib.DSA_ERR_ARG
    # unknown indexer-score flags are refused before anything runs
    assert L.dsa_indexer_score_ex(1, 1, 1, 1, None, 1, 64, 128, 8, 1024, 8, 4, None) == _lib.DSA_ERR_ARG
    assert "flags" in _lib.last_error()


def test_attention_rejects_row_count_overflow():
    from dsv4attn import _lib
    L = _lib.lib()
    B, S = 1 << 20, 1 << 12                      # B * S * 64 overflows a 32-bit row index
    assert L.dsa_sparse_attn_workspace_size(B, S, 64, 512, 2176) == 0
    rc = L.dsa_sparse_attn(16, 16, 512, 1, 16, 2176, 16, 16, None, B, S, 64, 512, 2176, 1.0, None, 0, None, None)
    assert rc == _lib.DSA_ERR_ARG and "too many" in _lib.last_error()
    rc = L.dsa_sparse_attn_noalloc(16, 16, 512, 1, 16, 2176, 16, 16, None, B, S, 64, 512, 2176, 1.0, None, None)
    assert rc == _lib.DSA_ERR_ARG and "too many" in _lib.last_error()


def test_workspace_queries_are_pure_host():
    from dsv4attn import _lib
    L = _lib.lib()
    assert L.dsa_indexer_topk_workspace_size(64, 8192, 2048) == 0
    assert L.dsa_indexer_topk_workspace_size(1, 65536, 2048) == 4 * 2048 * 8


def test_ops_refuse_cpu_tensors():
    import torch
    from dsv4attn import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.act_quant_block(torch.zeros(2, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        ops.sparse_attn(torch.zeros(1, 64, 512, dtype=torch.bfloat16), torch.zeros(1, 4, 512, dtype=torch.bfloat16),
                        torch.zeros(1, 4, dtype=torch.int32), torch.zeros(64), 0.1)


def test_bucket_picker_matches_reference_then_extends(golden):
    from dsv4attn.tables import pick_indexer_topk_bucket
    for t, want in zip(golden["bucket_t"], golden["bucket_pick"]):
        if t <= 1024:
            assert pick_indexer_topk_bucket(int(t)) == int(want)
    assert pick_indexer_topk_bucket(8192) == 8192
    assert pick_indexer_topk_bucket(8193) == 8320


def test_product_rope_tables_match_reference(golden):
    import numpy as np
    from dsv4attn.tables import PathArgs, rope_cos_sin
    rows = golden["freqs_rows"]
    c, s = rope_cos_sin(PathArgs(), int(rows.max()) + 1, compressed=True)
    np.testing.assert_allclose(c[rows].numpy(), golden["freqs_cmp_cos"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(s[rows].numpy(), golden["freqs_cmp_sin"], atol=2e-6, rtol=0)


def test_linear_packed_bytes_is_host_arithmetic():
    """The tile layout's size is G x ceil(N/128) x K/64 tiles of 16 KB; K not
    a multiple of 64 (or a non-positive size) gives 0."""
    from dsv4attn import _lib
    L = _lib.lib()
    assert L.dsa_linear_packed_bytes(128, 64, 1) == 16384
    assert L.dsa_linear_packed_bytes(200, 128, 1) == 2 * 2 * 16384
    assert L.dsa_linear_packed_bytes(1024, 4096, 8) == 8 * 8 * 64 * 16384
    assert L.dsa_linear_packed_bytes(64, 96, 1) == 0
    assert L.dsa_linear_packed_bytes(0, 64, 1) == 0
