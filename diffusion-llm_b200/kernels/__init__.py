"""Drop-in replacements for the reference's ``kernels/`` modules.

Same module names, function/class names and call signatures as
tusharsonthalia/diffusion-llm's kernels/BlockSparseFlashAttention.py,
kernels/SplitKVDecodeAttention.py and kernels/BlockSparseDecodeAttention.py, backed by the
hand-written sm_100a CUDA library (libbd3attn.so) instead of Triton. Put
``diffusion-llm_b200/`` on ``sys.path`` and the reference's model/bd3lm.py, model/kv_cache.py,
inference/generate.py and bench/attention_bench.py import these instead. (This is a regular
package, so it is chosen over the reference's namespace package of the same name wherever
the two sit on the path.)
"""
