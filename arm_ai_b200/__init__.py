"""arm_ai_b200 — B200 (sm_100a) implementation of arm_ai's quantized-Llama
decode path and its int8/int4 primitive NIFs.

The product is ``libarmai_cuda.so`` (C ABI in ``include/armai.h``); this
package holds its sources (``csrc/``), the in-tree build, and Python mirrors of
the reference's interfaces for this path:

  * ``llama_candle.LlamaCandle`` — ArmAI.LlamaCandle load / generate / stream
  * ``native`` — the llama_candle_*_op NIFs
  * ``prims`` — the int8/int4/rmsnorm/flash-attention primitive NIFs
  * ``synth`` — seeded random-init GGUF models for tests and benchmarks
"""
from .llama_candle import ArgumentError, LlamaCandle  # noqa: F401

__version__ = "0.1.0"
