"""kappa_b200 — B200-native (sm_100a) W8 fake-quant feed-forward path of kappa.

Drop-in replacements for kappa's W8 feed-forward functions, with kappa's
signatures, running on hand-written tcgen05 / TMA kernels behind the C ABI
in ``include/kappa_w8.h`` (``libkappa_w8.so``, built in-tree):

* ``kappa_b200.qwen3.quant``: ``Q8Weight``, ``quantize_weight``, ``to_compute_dtype``
* ``kappa_b200.gemma3.ffn.feed_forward`` (Gemma3 gated-GELU MLP)
* ``kappa_b200.qwen3.ffn.swiglu_ffn`` (Qwen3 dense SwiGLU)
* ``kappa_b200.qwen3.ffn_moe.moe_swiglu_ffn`` / ``moe_swiglu_ffn_legacy``
"""

__version__ = "0.1.0"
