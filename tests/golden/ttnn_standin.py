"""Test-only stand-in for the ``ttnn`` ops the reference's decode-path chains
call, with plain torch semantics.

TEST INFRASTRUCTURE ONLY: ``tests/golden/make_ref_chains.py`` installs it as
``sys.modules['ttnn']`` and then runs the reference's own functions
(``_device_act_quant_block``, ``DeviceAttention._indexer_topk_body``,
``DeviceSparseAttn.forward_device`` ...) on CPU tensors to produce golden
fixtures.  Nothing in the product path imports this file.

A "device tensor" here is just a torch tensor.  ``policy`` picks what the
reference's ``ttnn.bfloat16`` means: ``"fp32"`` keeps every float tensor in
float32, so a chain computes its published algorithm in fp32 arithmetic
(the precision this build computes in); ``"bf16"`` keeps bfloat16 as the
Tenstorrent device does.  Each op below is the torch operation with the same
name and argument meaning in ttnn's Python API; the ops nobody on the
reference's path calls are not provided, so an unexpected call fails loudly.
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F


class _Tok:
    """Named constant (layouts, memory configs, op types)."""

    def __init__(self, name: str):
        self.name = name

    def __repr__(self):
        return f"ttnn.{self.name}"


def make_ttnn(policy: str = "fp32") -> types.ModuleType:
    if policy not in ("fp32", "bf16"):
        raise ValueError(policy)
    m = types.ModuleType("ttnn")
    float_t = torch.float32 if policy == "fp32" else torch.bfloat16

    # ---- dtypes, layouts, memory configs
    m.bfloat16 = "bfloat16"
    m.float32 = "float32"
    m.int32 = "int32"
    m.uint32 = "uint32"
    m.uint16 = "uint16"
    m.TILE_LAYOUT = _Tok("TILE_LAYOUT")
    m.ROW_MAJOR_LAYOUT = _Tok("ROW_MAJOR_LAYOUT")
    m.DRAM_MEMORY_CONFIG = _Tok("DRAM_MEMORY_CONFIG")
    m.L1_MEMORY_CONFIG = _Tok("L1_MEMORY_CONFIG")
    m.UnaryOpType = types.SimpleNamespace(EXP=_Tok("UnaryOpType.EXP"))

    def tdtype(d):
        if d is None:
            return None
        if isinstance(d, torch.dtype):
            return float_t if d.is_floating_point else d
        return {"bfloat16": float_t, "float32": torch.float32, "int32": torch.int32,
                "uint32": torch.int64, "uint16": torch.int64}[d]

    def as_t(x, like=None):
        if isinstance(x, torch.Tensor):
            return x
        dt = like.dtype if isinstance(like, torch.Tensor) else float_t
        return torch.tensor(x, dtype=dt)

    # ---- host <-> "device"
    def from_torch(t, dtype=None, layout=None, device=None, memory_config=None, mesh_mapper=None, **_):
        out = t.detach().clone()
        dt = tdtype(dtype) if dtype is not None else (float_t if out.is_floating_point() else out.dtype)
        return out.to(dt)

    m.from_torch = from_torch
    m.as_tensor = from_torch
    m.to_torch = lambda t, mesh_composer=None, **_: t
    m.ReplicateTensorToMesh = lambda *a, **k: None
    m.ShardTensor2dMesh = lambda *a, **k: None
    m.ConcatMesh2dToTensor = lambda *a, **k: None

    def zeros(shape, dtype=None, layout=None, device=None, memory_config=None, **_):
        return torch.zeros(tuple(shape), dtype=tdtype(dtype) or float_t)

    m.zeros = zeros
    m.Shape = lambda s: tuple(s)

    # ---- shape ops
    m.reshape = lambda t, shape, **_: t.reshape(tuple(shape))
    m.to_layout = lambda t, layout, **_: t

    def slice_(t, starts, ends, steps=None, **_):
        return t[tuple(slice(int(a), int(b)) for a, b in zip(starts, ends))].clone()

    m.slice = slice_
    m.concat = lambda ts, dim=0, **_: torch.cat(list(ts), dim=dim)
    m.transpose = lambda t, d0, d1, **_: t.transpose(d0, d1)
    m.repeat = lambda t, shape, **_: t.repeat(*tuple(shape))

    def pad(t, padding, value=0.0, **_):
        flat = []
        for lo, hi in reversed(list(padding)):
            flat += [int(lo), int(hi)]
        return F.pad(t, flat, value=value)

    m.pad = pad

    # ---- elementwise
    m.abs = lambda t, **_: t.abs()
    m.relu = lambda t, **_: torch.relu(t)
    m.rsqrt = lambda t, **_: torch.rsqrt(t)
    m.clamp = lambda t, min=None, max=None, **_: torch.clamp(t, min=min, max=max)

    def maximum(a, b, **_):
        return torch.maximum(a, as_t(b, a))

    m.maximum = maximum

    def multiply(a, b, **_):
        return a * b

    m.multiply = multiply

    def divide(a, b, **_):
        return a / b

    m.divide = divide

    def add(a, b, dtype=None, **_):
        out = a + b
        return out.to(tdtype(dtype)) if dtype is not None else out

    m.add = add

    def subtract(a, b, activations=None, **_):
        out = a - b
        for act in activations or []:
            if act is m.UnaryOpType.EXP:
                out = torch.exp(out)
            else:
                raise NotImplementedError(f"activation {act}")
        return out

    m.subtract = subtract

    def addcmul(a, b, c, value=1.0, **_):
        return a + value * (b * c)

    m.addcmul = addcmul

    def where(cond, x, y, **_):
        c = cond.bool() if cond.dtype != torch.bool else cond
        xt = x if isinstance(x, torch.Tensor) else torch.tensor(x, dtype=float_t)
        yt = y if isinstance(y, torch.Tensor) else torch.tensor(y, dtype=float_t)
        return torch.where(c, xt, yt)

    m.where = where

    def _cmp(op):
        def f(a, b, dtype=None, **_):
            r = op(a, as_t(b, a))
            return r.to(tdtype(dtype) if dtype is not None else a.dtype)
        return f

    m.lt = _cmp(torch.lt)
    m.gt = _cmp(torch.gt)
    m.ge = _cmp(torch.ge)
    m.le = _cmp(torch.le)
    m.eq = _cmp(torch.eq)
    m.typecast = lambda t, dtype, **_: t.to(tdtype(dtype))

    # ---- reductions / contractions
    def max_(t, dim=None, keepdim=False, **_):
        return t.amax(dim=dim, keepdim=keepdim)

    m.max = max_
    m.sum = lambda t, dim=None, keepdim=False, **_: t.sum(dim=dim, keepdim=keepdim)
    m.mean = lambda t, dim=None, keepdim=False, **_: t.mean(dim=dim, keepdim=keepdim)
    m.softmax = lambda t, dim=-1, **_: torch.softmax(t, dim=dim)

    def matmul(a, b, transpose_a=False, transpose_b=False, **_):
        if transpose_a:
            a = a.transpose(-1, -2)
        if transpose_b:
            b = b.transpose(-1, -2)
        return torch.matmul(a, b)

    m.matmul = matmul

    def topk(t, k, dim=-1, largest=True, sorted=True, **_):
        v, i = torch.topk(t, int(k), dim=dim, largest=largest, sorted=sorted)
        return v, i.to(torch.int64)

    m.topk = topk

    def embedding(idx, table, layout=None, **_):
        return table[idx.long()]

    m.embedding = embedding

    def copy(src, dst, **_):
        dst.copy_(src)
        return dst

    m.copy = copy

    # ---- in-place cache updates
    def update_cache_for_token_(cache, x, idx, batch_offset=0):
        # cache [B, 1, T, d] <- x [B, 1, 1, d] at slot idx
        cache[:, :, int(idx):int(idx) + 1] = x.to(cache.dtype)

    m.kv_cache = types.SimpleNamespace(update_cache_for_token_=update_cache_for_token_)
    return m


class AnyStub(types.ModuleType):
    """Stands in for modules only touched at import time (``ttl``): every
    attribute is itself, and calling it with a function returns that
    function (decorator use)."""

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return self

    def __call__(self, *args, **kwargs):
        if args and callable(args[0]) and not kwargs:
            return args[0]
        return self
