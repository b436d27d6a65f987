"""CPU oracle for the DeepSeek-V4-Flash decode sparse-attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package may import this
module: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline legs use it, and only as the checker / the timed CPU baseline.

The oracle is a plain-torch (fp32, CPU) restatement of the reference's
per-layer decode path (zoecarver/tt-deepseek-v4, ``inference.py``), stage by
stage, each function citing the reference lines it follows.  See
``oracle/path.py``.

Parity pinning: the reference's own CPU forward passes were deleted from
``inference.py`` and its device path needs ttnn/tt-lang/Tenstorrent hardware,
so the path cannot be executed here end to end.  The oracle is pinned in two
ways (tests/test_oracle_*.py):

* against the reference's surviving pure-torch helpers, imported from the
  reference with a stub ``ttl`` module by ``tests/golden/make_golden.py``
  (window-index table, slot-shift matrix, softmax-sum-norm masks, YaRN
  ``precompute_freqs_cis``, rotary swap tables, Hadamard matrix, top-k
  bucket picker) - committed as ``tests/golden/ref_helpers.npz``;
* against hand-computable known answers taken from the reference's
  docstrings and ttnn op chains (one-hot scores for top-k, equal gates for
  the compressor softmax, a single valid index for sparse attention, values
  on the e4m3 grid for act_quant).

The ttnn arithmetic itself (``ttnn.topk``, ``ttnn.matmul``...) is not pinned
against the library (tt-metal is not vendored, its version is unpinned):
parity is "partially pinned" in that sense.
"""

from .path import *  # noqa: F401,F403
