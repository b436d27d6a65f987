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
so the path cannot be executed here end to end on its device.  The oracle is
pinned in three ways (tests/test_oracle_*.py):

* against the reference's own device op chains - ``_device_act_quant_block``,
  ``DeviceAttention._indexer_topk_body`` and the verbatim chain of
  tt-lang-kernels/mega/test_lk_d_topk.py, ``DeviceSparseAttn.forward_device``,
  the indexer score reference, ``DeviceCompressorOverlap`` /
  ``DeviceCompressorNoOverlap`` - run unmodified on CPU through a test-only
  torch stand-in for ``ttnn`` (fp32 policy) by
  ``tests/golden/make_ref_chains.py``, committed as
  ``tests/golden/ref_chains.npz``;
* against the reference's surviving pure-torch helpers, imported from the
  reference with a stub ``ttl`` module by ``tests/golden/make_golden.py``
  (window-index table, slot-shift matrix, softmax-sum-norm masks, YaRN
  ``precompute_freqs_cis``, rotary swap tables, Hadamard matrix, top-k
  bucket picker) - committed as ``tests/golden/ref_helpers.npz``;
* against hand-computable known answers taken from the reference's
  docstrings and ttnn op chains (one-hot scores for top-k, equal gates for
  the compressor softmax, a single valid index for sparse attention, values
  on the e4m3 grid for act_quant).

What stays unpinned is the Tenstorrent device arithmetic itself
(``ttnn.topk``'s tie order, bf16 device rounding): the chain fixtures are the
reference's algorithms evaluated in fp32 on bf16-valued inputs.
"""

from .path import *  # noqa: F401,F403
