"""Generate tests/golden/ref_chains.npz by running the reference's OWN decode
path functions on CPU through the torch stand-in for ttnn.

Run in a container where the reference checkout is available:

    python tests/golden/make_ref_chains.py REFERENCE_DIR

The reference's device code calls ``ttnn`` ops; ``ttnn_standin.make_ttnn``
gives each op its torch meaning, so the reference functions below run
unmodified and their outputs become fixtures.  Policy "fp32": every float
tensor the reference would hold in bfloat16 is held in float32, i.e. the
fixtures are the reference's algorithms evaluated in fp32 arithmetic on
bf16-valued inputs (the precision this build computes in).  The chains:

* ``_device_act_quant_block`` (inference.py:4578-4607), with the scale
  ``multiply(amax, 1/fp8_max)`` captured from inside the chain;
* ``DeviceAttention._indexer_topk_body`` (inference.py:5823-5851) on buffers
  built as ``_alloc_decode_tensors`` builds them (5544-5600), and the
  verbatim reference chain ``_indexer_topk_body_ref``
  (tt-lang-kernels/mega/test_lk_d_topk.py:121-138);
* ``DeviceSparseAttn._idxs_int_tile_to_idxs_and_mask`` + ``forward_device``
  (inference.py:4444-4501);
* the indexer score reference (tt-lang-kernels/mega/test_lk_d_idx_score.py:359-371);
* ``DeviceCompressorOverlap.forward_device`` and
  ``DeviceCompressorNoOverlap.forward_device``
  (device-compressor-indexer/compressor_overlap.py, compressor_no_overlap.py)
  over several decode steps.  Those classes call the rotary stub
  ``_device_apply_rotary_interleaved`` (which raises by design,
  inference.py:4556-4564) and a tt-lang RMSNorm; the script substitutes the
  reference's live rotary ``_device_apply_rotary_swap`` on tables from
  ``_build_rotary_aux_tables`` / ``_build_rotary_swap_matrix``
  (inference.py:4504-4553) and the reference's CPU ``RMSNorm`` module
  (inference.py:438-450).

The GPU box never runs this script: the tests only read the ``.npz``.
"""

from __future__ import annotations

import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from ttnn_standin import AnyStub, make_ttnn  # noqa: E402


def install(ref_dir: str, policy: str = "fp32"):
    tt = make_ttnn(policy)
    sys.modules["ttnn"] = tt
    sys.modules["ttl"] = AnyStub("ttl")
    for p in (ref_dir, os.path.join(ref_dir, "tt-lang-kernels", "mega"),
              os.path.join(ref_dir, "device-compressor-indexer")):
        if p not in sys.path:
            sys.path.insert(0, p)
    I = importlib.import_module("inference")
    return tt, I


def bf16(t: torch.Tensor) -> torch.Tensor:
    """bf16-valued fp32 tensor (the values the reference uploads)."""
    return t.to(torch.bfloat16).float()


def chain_act_quant(tt, I, g, out):
    rows = [torch.randn(24, 448, generator=g)]
    rows.append(torch.randn(4, 448, generator=g) * 1e-3)
    rows.append(torch.randn(4, 448, generator=g) * 300.0)
    rows.append(torch.zeros(1, 448))                                   # amax 0 -> eps floor
    rows.append(torch.full((1, 448), 3e-6))                            # amax below eps
    e4 = torch.tensor([0.0, 0.001953125, 0.5, 1.0, 1.125, 448.0, -448.0, 240.0], dtype=torch.float32)
    rows.append(e4.repeat(56).view(1, 448))                            # values on the e4m3 grid
    spike = torch.randn(1, 448, generator=g) * 0.01
    spike[0, 7] = 40.0
    rows.append(spike)
    x = bf16(torch.cat(rows))
    taps = []
    mul = tt.multiply

    def tap(a, b, **kw):
        r = mul(a, b, **kw)
        taps.append(r.clone())
        return r

    tt.multiply = tap
    y = I._device_act_quant_block(tt, x.clone(), 64)
    tt.multiply = mul
    out["aq_x"] = x.numpy()
    out["aq_out"] = y.numpy()                 # clamp(x / s) * s, fp32, no e4m3 cast
    out["aq_scale"] = taps[0].squeeze(-1).numpy()   # multiply(amax, 1 / fp8_max): [rows, 7]


def chain_topk(tt, I, g, out):
    """DeviceAttention._indexer_topk_body on the buffers of _alloc_decode_tensors."""
    cases = []
    # (bucket, index_topk, win, per-batch T_active, score kind)
    cases.append((128, 64, 128, [50, 128, 3], "randn"))
    cases.append((256, 128, 128, [200, 256, 130], "randn"))
    cases.append((1024, 512, 128, [1024, 700, 511], "randn"))
    cases.append((512, 512, 128, [300, 512, 17], "ties"))
    for ci, (bk, index_topk, win, t_act, kind) in enumerate(cases):
        B, S = len(t_act), 1
        if kind == "randn":
            score = torch.randn(B, S, bk, generator=g)
        else:
            score = torch.randint(-6, 7, (B, S, bk), generator=g).float() * 0.25
        k_fixed = min(index_topk, bk)
        self = types.SimpleNamespace(_ttnn=tt)
        self._indexer_score_in_tt = tt.from_torch(score, dtype=tt.bfloat16)
        ramp = torch.arange(bk, dtype=torch.int32).view(1, 1, bk).expand(B, 1, bk).contiguous()
        self._topk_ramp_int_per_bucket = {bk: tt.from_torch(ramp, dtype=tt.int32)}
        ta = torch.tensor(t_act, dtype=torch.int32).view(B, 1, 1).expand(B, 1, bk).contiguous()
        self._t_active_persistent_per_bucket = {bk: tt.from_torch(ta, dtype=tt.int32)}
        self._topk_neg_const_per_bucket = {bk: tt.from_torch(torch.full((B, 1, bk), -1e4, dtype=torch.bfloat16),
                                                             dtype=tt.bfloat16)}
        self._topk_neg_one_int_per_bucket = {k_fixed: tt.from_torch(torch.full((B, 1, k_fixed), -1, dtype=torch.int32),
                                                                    dtype=tt.int32)}
        res = I.DeviceAttention._indexer_topk_body(self, bk, k_fixed, win, B, S)
        out[f"tk{ci}_score"] = score.numpy()
        out[f"tk{ci}_t_active"] = np.array(t_act, dtype=np.int32)
        out[f"tk{ci}_meta"] = np.array([bk, k_fixed, win], dtype=np.int32)
        out[f"tk{ci}_idx"] = res.to(torch.int32).numpy()
    out["tk_cases"] = np.array(len(cases))

    # the verbatim reference chain of the Lk-D-topk test, at its own shapes
    T = importlib.import_module("test_lk_d_topk")
    score = bf16(torch.randn(1, 1, T.T_PAD, generator=g))
    ramp = torch.arange(T.BUCKET, dtype=torch.int32).view(1, 1, T.BUCKET)
    t_active = torch.full((1, 1, T.BUCKET), 50, dtype=torch.int32)
    res = T._indexer_topk_body_ref(tt.from_torch(score, dtype=tt.bfloat16), tt.from_torch(ramp, dtype=tt.int32),
                                   tt.from_torch(t_active, dtype=tt.int32))
    out["tkref_score"] = score.numpy()
    out["tkref_meta"] = np.array([T.BUCKET, T.K_FIXED, T.WIN, 50], dtype=np.int32)
    out["tkref_idx"] = res.to(torch.int32).numpy()


def chain_sparse_attn(tt, I, g, out):
    """DeviceSparseAttn._idxs_int_tile_to_idxs_and_mask + forward_device."""
    H, D, N, K, S = 64, 512, 300, 96, 3
    q = bf16(torch.randn(1, S, H, D, generator=g) * (D ** -0.5))     # softmax_scale pre-baked into q
    kv = bf16(torch.randn(N, D, generator=g))
    idx = torch.randint(0, N, (1, S, K), generator=g, dtype=torch.int32)
    idx[0, 0, 70:] = -1                                                # masked tail
    idx[0, 1, ::7] = -1                                                # scattered holes
    idx[0, 2, :] = -1                                                  # nothing valid: sink only
    sink = bf16(torch.randn(H, generator=g))
    self = types.SimpleNamespace(_ttnn=tt, n_heads=H)
    self.sink_tt = tt.as_tensor(sink.view(1, 1, H, 1), dtype=tt.bfloat16)
    safe, valid = I.DeviceSparseAttn._idxs_int_tile_to_idxs_and_mask(self, tt.from_torch(idx, dtype=tt.int32), 1, S, K)
    o = I.DeviceSparseAttn.forward_device(self, tt.from_torch(q, dtype=tt.bfloat16), tt.from_torch(kv, dtype=tt.bfloat16),
                                          safe, valid, S, K)
    out["sa_q"] = q.numpy()
    out["sa_kv"] = kv.numpy()
    out["sa_idx"] = idx.numpy()
    out["sa_sink"] = sink.numpy()
    out["sa_safe"] = safe.to(torch.int64).numpy()
    out["sa_valid"] = valid.numpy()
    out["sa_out"] = o.numpy()


def chain_idx_score(tt, I, g, out):
    """The indexer score reference chain of the Lk-D-idx-score test."""
    T = importlib.import_module("test_lk_d_idx_score")
    dim, H, Dh, Tn = 256, T.INDEX_N_HEADS, T.INDEX_HEAD_DIM, T.T_PAD
    x = bf16(torch.randn(1, 1, dim, generator=g) * 0.1)
    wproj = bf16(torch.randn(dim, H, generator=g) * 0.02)
    q_idx = bf16(torch.randn(1, 1, H, Dh, generator=g) * 0.1)
    kv = bf16(torch.randn(1, 1, Tn, Dh, generator=g) * 0.1)
    scale = float(Dh ** -0.5) * float(H ** -0.5)
    s = T.reference(None, x, wproj, q_idx, kv, scale)
    out["is_x"], out["is_wproj"], out["is_q"], out["is_kv"] = x.numpy(), wproj.numpy(), q_idx.numpy(), kv.numpy()
    out["is_scale"] = np.array(scale, dtype=np.float64)
    out["is_out"] = s.numpy()


class _Lin:
    """Stands in for the on-device wkv / wgate linear: returns the next
    pre-drawn output row of this step."""

    def __init__(self):
        self.rows = []

    def forward_device(self, x_tt):
        return self.rows.pop(0)


class _Norm:
    """The reference's CPU RMSNorm module standing in for the tt-lang one."""

    def __init__(self, norm):
        self.norm = norm

    def forward_device(self, x, B):
        with torch.no_grad():
            return self.norm(x)


def chain_compressors(tt, I, g, out):
    from harness import make_test_args

    def rotary_interleaved(ttnn, x, cos, sin, inverse=False):
        cos_ext, sin_signed = I._build_rotary_aux_tables(cos, sin)
        P = I._build_rotary_swap_matrix(x.shape[-1], dtype=torch.float32)
        return I._device_apply_rotary_swap(ttnn, x, cos_ext, sin_signed, P, inverse=inverse)

    I._device_apply_rotary_interleaved = rotary_interleaved
    args = make_test_args(I, max_seq_len=64)
    args.max_batch_size = 2
    for name, ratio, mod, cls, steps in (("co", 4, "compressor_overlap", "DeviceCompressorOverlap", 13),
                                         ("cn", 8, "compressor_no_overlap", "DeviceCompressorNoOverlap", 25)):
        M = importlib.import_module(mod)
        M.inf._device_apply_rotary_interleaved = rotary_interleaved
        comp = M.inf.Compressor(args, compress_ratio=ratio, head_dim=512, rotate=False).eval()
        with torch.no_grad():
            comp.ape.copy_(torch.randn(comp.ape.shape, generator=g))
            comp.norm.weight.copy_(1.0 + 0.02 * torch.randn(512, generator=g))
        comp.kv_cache = torch.zeros(args.max_batch_size, args.max_seq_len // ratio, 512)
        comp.freqs_cis = M.inf.precompute_freqs_cis(comp.rope_head_dim, args.max_seq_len, args.original_seq_len,
                                                    args.compress_rope_theta, args.rope_factor, args.beta_fast,
                                                    args.beta_slow)
        wkv, wgate = _Lin(), _Lin()
        dc = getattr(M, cls)(types.SimpleNamespace(shape=(1, 1)), comp, wkv, wgate, _Norm(comp.norm))
        B = args.max_batch_size
        c = comp.ape.shape[1]
        kv_in = bf16(torch.randn(steps, B, 1, c, generator=g))
        sc_in = bf16(torch.randn(steps, B, 1, c, generator=g))
        emits = np.zeros((steps, B, 512), dtype=np.float32)
        emitted = np.zeros(steps, dtype=np.int32)
        for pos in range(steps):
            wkv.rows.append(kv_in[pos].clone())
            wgate.rows.append(sc_in[pos].clone())
            r = dc.forward_device(None, B, pos)
            if r is not None:
                emits[pos] = r.reshape(B, 512).numpy()
                emitted[pos] = 1
        out[f"{name}_ratio"] = np.array(ratio)
        out[f"{name}_kv_in"] = kv_in.numpy()
        out[f"{name}_sc_in"] = sc_in.numpy()
        out[f"{name}_ape"] = bf16(comp.ape.detach()).numpy()           # uploaded bf16
        out[f"{name}_gamma"] = comp.norm.weight.detach().numpy()
        out[f"{name}_cos"] = bf16(comp.freqs_cis.real).numpy()
        out[f"{name}_sin"] = bf16(comp.freqs_cis.imag).numpy()
        out[f"{name}_emits"] = emits
        out[f"{name}_emitted"] = emitted
        out[f"{name}_cache"] = dc.kv_cache_tt.reshape(B, -1, 512)[:, : args.max_seq_len // ratio].numpy()
        if ratio == 4:
            kvs, scs = M._gather_cpu_state(dc, B)
        else:
            rp = dc.ratio_pad
            kvs = dc.kv_state_tt.reshape(B, rp, 512)[:, :ratio]
            scs = dc.score_state_tt.reshape(B, rp, 512)[:, :ratio]
        out[f"{name}_kv_state"] = kvs.numpy()
        out[f"{name}_sc_state"] = scs.numpy()


def main(ref_dir: str, out_path: str) -> None:
    tt, I = install(ref_dir, "fp32")
    g = torch.Generator().manual_seed(20261202)
    out: dict[str, np.ndarray] = {}
    chain_act_quant(tt, I, g, out)
    chain_topk(tt, I, g, out)
    chain_sparse_attn(tt, I, g, out)
    chain_idx_score(tt, I, g, out)
    chain_compressors(tt, I, g, out)
    np.savez_compressed(out_path, **out)
    print(f"wrote {out_path}: {len(out)} arrays, {os.path.getsize(out_path) / 1e6:.2f} MB")


if __name__ == "__main__":
    if len(sys.argv) > 1:
        ref = sys.argv[1]
    elif "DSV4_REFERENCE_DIR" in os.environ:
        ref = os.environ["DSV4_REFERENCE_DIR"]
    else:
        sys.exit("usage: make_ref_chains.py REFERENCE_DIR  (or set DSV4_REFERENCE_DIR)")
    main(ref, os.path.join(HERE, "ref_chains.npz"))
