"""Generate tests/golden/ref_helpers.npz from the reference's own helpers.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py [REFERENCE_DIR]

It imports the reference's ``inference.py`` with a stub ``ttl`` module (the
tt-lang DSL is not installed; only its decorators are touched at import time)
and records the outputs of the pure-torch helpers that define the path's
index, rotary and state-shift conventions.  The GPU box never runs this
script: the tests only read the committed ``.npz``.
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch


class _AnyStub(types.ModuleType):
    """Stands in for the ``ttl`` package: every attribute is itself, and
    calling it with a function returns that function (decorator use)."""

    def __getattr__(self, name):
        return self

    def __call__(self, *args, **kwargs):
        if args and callable(args[0]) and not kwargs:
            return args[0]
        return self


def load_reference(ref_dir: str):
    sys.modules.setdefault("ttl", _AnyStub("ttl"))
    sys.path.insert(0, ref_dir)
    import inference  # noqa: E402
    return inference


def main(ref_dir: str, out_path: str) -> None:
    I = load_reference(ref_dir)
    g = torch.Generator().manual_seed(1234)
    out: dict[str, np.ndarray] = {}

    # window-index table and its per-position row picker (inference.py:479-506)
    for win in (4, 8, 128):
        out[f"window_table_{win}"] = I._build_window_topk_table(win).numpy()
    pos = np.array([0, 1, 5, 126, 127, 128, 129, 255, 256, 1000, 4095, 32767, 32770], dtype=np.int64)
    out["window_row_pos"] = pos
    out["window_row_128"] = np.array([I._window_topk_row_for_pos(int(p), 128) for p in pos])

    # indexer top-k buckets (inference.py:509-520)
    t = np.arange(1, 1101)
    out["bucket_t"] = t
    out["bucket_pick"] = np.array([I._pick_indexer_topk_bucket(int(x)) for x in t])

    # slot-shift matrix and its action on a random state (inference.py:3189-3202)
    P = I._compressor_shift_matrix(4, 32).float()
    out["shift_P_4_32"] = P.numpy()
    state = torch.randn(32, 16, generator=g)
    out["shift_in"] = state.numpy()
    out["shift_out"] = (P @ state).numpy()

    # softmax-sum-norm masks (inference.py:3367-3380)
    mf, mb, mp = I._compressor_softmax_sum_norm_masks(4)
    out["cssn_mf"], out["cssn_mb"], out["cssn_mp"] = mf.float().numpy(), mb.float().numpy(), mp.float().numpy()

    # YaRN rotary tables (inference.py:453-476): compressed layers use
    # original_seq_len 65536, theta 160000; dense layers theta 10000, no YaRN.
    rows = np.array([0, 1, 2, 3, 127, 128, 4095, 32767, 65535, 131071, 262143], dtype=np.int64)
    out["freqs_rows"] = rows
    fc = I.precompute_freqs_cis(64, 262144, 65536, 160000.0, 16, 32, 1)
    out["freqs_cmp_cos"] = fc.real[rows].numpy()
    out["freqs_cmp_sin"] = fc.imag[rows].numpy()
    fd = I.precompute_freqs_cis(64, 262144, 0, 10000.0, 16, 32, 1)
    out["freqs_dense_cos"] = fd.real[rows].numpy()
    out["freqs_dense_sin"] = fd.imag[rows].numpy()

    # rotary convention via the reference's swap-matrix form (4504-4553)
    x = torch.randn(6, 64, generator=g)
    cos_ext, sin_signed = I._build_rotary_aux_tables(fc.real[rows[:6]].float(), fc.imag[rows[:6]].float())
    Psw = I._build_rotary_swap_matrix(64, dtype=torch.float32)
    out["rot_x"] = x.numpy()
    out["rot_rows"] = rows[:6]
    out["rot_out"] = (x * cos_ext + (x @ Psw) * sin_signed).numpy()
    out["rot_inv_out"] = (x * cos_ext - (x @ Psw) * sin_signed).numpy()

    # Hadamard rotation used by the indexer compressor (inference.py:4610-4631)
    H = I._sylvester_hadamard(128) * (128 ** -0.5)
    xh = torch.randn(3, 128, generator=g)
    out["had_x"] = xh.numpy()
    out["had_out"] = (xh @ H).numpy()

    # compressor state initialisation and shapes (inference.py:523-552)
    args = I.ModelArgs(max_batch_size=2, max_seq_len=64)
    comp = I.Compressor(args, 4, 512)
    out["cmp_kv_state"] = comp.kv_state.numpy()
    out["cmp_score_state"] = comp.score_state.numpy()
    comp128 = I.Compressor(args, 128, 512)
    out["cmp128_state_shape"] = np.array(comp128.kv_state.shape)
    attn = I.Attention(2, args)
    out["attn_kv_cache_shape"] = np.array(attn.kv_cache.shape)
    out["attn_softmax_scale"] = np.array(attn.softmax_scale)
    out["index_topk"] = np.array(args.index_topk)

    np.savez_compressed(out_path, **out)
    print(f"wrote {out_path}: {len(out)} arrays")


if __name__ == "__main__":
    if len(sys.argv) > 1:
        ref = sys.argv[1]
    elif "DSV4_REFERENCE_DIR" in os.environ:
        ref = os.environ["DSV4_REFERENCE_DIR"]
    else:
        sys.exit("usage: make_golden.py REFERENCE_DIR  (or set DSV4_REFERENCE_DIR)")
    here = os.path.dirname(os.path.abspath(__file__))
    main(ref, os.path.join(here, "ref_helpers.npz"))
