"""CPU oracle for the routed-expert MoE path and the quantized KV-cache formats.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (``whallm_b200``)
imports, links or executes this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm use it, and
only as the checker (or as the timed CPU restatement).

The reference (baha2046/Whallm) computes this path with MLX library calls
(``mlx==0.32.2``, ``mlx-lm@5c10538``) that are not vendored and cannot run
here.  The oracle restates, in numpy and plain C:

* ``formats``  -- MXFP4 quantize (``Sources/DeepSeekRepack/MXFP4.swift:4-131``),
  MXFP4/E8M0 dequant (``runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:24-66``),
  the packed KV row formats (``deepseek_v41/packed_cache.py:24-59`` with
  ``deepseek_v41/fakequant.py:47-119``), the per-64 fp32-scale FP8 KV format,
  and MLX-style affine 4-bit (parity unpinned, see ``formats.affine4_quantize``).
* ``router``   -- gate logits, score functions, top-k with the positional
  tie rule (``model.py:548-560``), renormalisation (``deepseek_v41/moe.py:58-75``,
  ``qwen4_exp.py:693-697``), evaluated in the same fixed fp32 order as the
  device kernel (via ``oracle/c/router_ref.c``), so indices compare exactly.
* ``moe``      -- the MoE layer composition (``model.py:393-504``,
  ``deepseek_v41/moe.py:30-112``, ``qwen4_exp.py:588-704``).
* ``loader``   -- the expert-slot layouts of an installed model and the
  region-by-region blob store (``expert_layout.py:8-80``,
  ``expert_cache.py:416-493``).

Pinning: ``formats`` is pinned by the reference's own known-answer tests
(``Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:336-411``) and by the
packed-cache == fake-quant identity (``runtime/tests/test_v41_packed_cache.py:12-26``);
see ``tests/test_oracle_pins.py``.
"""
