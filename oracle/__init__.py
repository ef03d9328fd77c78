"""CPU restatement of the ERNIE 5.5 HCA layer path -- TEST INFRASTRUCTURE ONLY.

This package is the parity oracle for the CUDA path in ``vllm-ernie_b200``.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker (or as the timed CPU baseline),
never as the thing measured or shipped.  The product path never falls back
to it.

Every function cites the reference file:line it restates.  Citation
prefixes:

* ``E/``  = ``src/vllm_ernie/models/ernie5_5/`` of baidu/vLLM-ERNIE (the plugin)
* ``V/``  = the vLLM package the plugin subclasses (``vllm/``).  The plugin
  pins vLLM 0.32.0; the readable sources used here are vLLM 0.22.0's, whose
  DeepSeek-V4 HCA arithmetic the plugin inherits.

Parity pin: integer builders, the KV-cache insert, compressor, dequant
gather, inverse-RoPE/FP8 quant and the plugin's own VHA and gate-quant
kernels are pinned against golden vectors produced by running the
reference's own Triton kernels under Triton's CPU interpreter
(``tests/golden/make_golden.py``).  The sparse attention core (FlashMLA)
exists only as a closed binary; its oracle follows the documented
semantics in ``V/third_party/flashmla/flash_mla_interface.py:54-92,180-215``
and is not pinned by a reference run.
"""
