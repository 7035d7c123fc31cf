"""ctypes bindings of libarmai_cuda.so (include/armai.h) and libarmai_synth.so.

The CUDA library is required: there is no CPU fallback. Loading fails loudly
when the library has not been built (``python -m arm_ai_b200.build``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import (POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int32, c_int64,
                    c_size_t, c_uint16, c_uint32, c_uint64, c_void_p)

PKG = os.path.dirname(os.path.abspath(__file__))
CUDA_LIB = os.path.join(PKG, "libarmai_cuda.so")
SYNTH_LIB = os.path.join(PKG, "libarmai_synth.so")

ARMAI_OK = 0
ERRORS = {-1: "invalid argument", -2: "io", -3: "format", -4: "cuda", -5: "out of memory",
          -6: "device error", -7: "range"}


class LlamaOpts(Structure):
    _fields_ = [("device", c_int32), ("max_seq_len", c_int32), ("kv_f16", c_int32),
                ("max_batch", c_int32), ("use_graph", c_int32), ("use_pdl", c_int32),
                ("tp_size", c_int32), ("tp_rank", c_int32), ("tp_unique_id", c_void_p),
                ("decode_kernel", c_int32), ("prefill_gemm", c_int32), ("batch_gemm", c_int32),
                ("reserved", c_int32 * 5)]


class LlamaInfo(Structure):
    _fields_ = [("n_layer", c_int32), ("n_embd", c_int32), ("n_ff", c_int32), ("n_head", c_int32),
                ("n_head_kv", c_int32), ("head_dim", c_int32), ("n_vocab", c_int32),
                ("max_seq_len", c_int32), ("rms_eps", c_float), ("rope_theta", c_float),
                ("weight_bytes", c_int64), ("device_bytes", c_int64),
                ("n_kernels_per_step", c_int32), ("kv_f16", c_int32)]


TOKEN_CB = ctypes.CFUNCTYPE(None, c_void_p, c_uint32)

_SIGS = {
    "armai_llama_default_opts": (None, [POINTER(LlamaOpts)]),
    "armai_llama_load": (c_int, [c_char_p, POINTER(LlamaOpts), POINTER(c_void_p)]),
    "armai_llama_free": (None, [c_void_p]),
    "armai_llama_get_info": (c_int, [c_void_p, POINTER(LlamaInfo)]),
    "armai_llama_generate": (c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p, c_size_t,
                                     TOKEN_CB, c_void_p, c_void_p, POINTER(c_size_t),
                                     POINTER(c_uint64), POINTER(c_uint64)]),
    "armai_llama_generate_batch": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_size_t,
                                           c_void_p, c_size_t, c_void_p, c_void_p,
                                           POINTER(c_uint64), POINTER(c_uint64)]),
    "armai_llama_forward": (c_int, [c_void_p, c_void_p, c_size_t, c_size_t, c_void_p,
                                    POINTER(c_uint32)]),
    "armai_llama_bench_decode": (c_int, [c_void_p, c_int32, POINTER(c_float)]),
    "armai_llama_bench_kernel": (c_int, [c_void_p, c_int32, c_int32, POINTER(c_float), POINTER(c_int64)]),
    "armai_llama_trace_decode": (c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_int32), POINTER(c_int32)]),
    "armai_llama_test_stall": (c_int, [c_void_p, c_int32, c_uint32]),
    "armai_int8_matmul_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                      c_double, c_size_t, c_size_t, c_size_t, c_void_p]),
    "armai_int8_matmul_f32_per_token": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p,
                                                c_size_t, c_void_p, c_size_t, c_size_t, c_size_t,
                                                c_size_t, c_void_p]),
    "armai_int8_matmul_s32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_size_t,
                                      c_size_t, c_void_p]),
    "armai_quantize_int8_per_token": (c_int, [c_void_p, c_size_t, c_size_t, c_size_t, c_void_p,
                                              c_void_p]),
    "armai_int4_matmul_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                      c_size_t, c_size_t, c_size_t, c_void_p]),
    "armai_int4_matmul_gemv": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                       c_size_t, c_size_t, c_void_p]),
    "armai_int4_matmul_gemv_q4_x_q8": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p,
                                               c_size_t, c_size_t, c_size_t, c_void_p]),
    "armai_quantize_int4_q4_0": (c_int, [c_void_p, c_size_t, c_size_t, c_size_t, c_void_p, c_void_p]),
    "armai_rmsnorm_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_size_t,
                                  c_double, c_void_p]),
    "armai_flash_attention_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                          c_double, c_size_t, c_size_t, c_size_t, c_size_t, c_size_t,
                                          c_int, c_void_p]),
    "armai_dequant_matmul_int8_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p,
                                              c_size_t, c_size_t, c_size_t, c_size_t, c_size_t,
                                              c_void_p]),
    "armai_rope_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t, c_size_t,
                               c_size_t, c_size_t, c_void_p]),
    "armai_dequant_matmul_f16_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_size_t, c_size_t,
                                             c_size_t, c_size_t, c_void_p]),
    "armai_softmax_last_axis_f32": (c_int, [c_void_p, c_size_t, c_size_t, c_size_t, c_void_p]),
    "armai_silu_gate_mul_up_f32": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t, c_void_p]),
    "armai_dequantize_q6_k": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p]),
    "armai_dev_rope_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                   c_void_p]),
    "armai_dev_softmax_last_axis_f32": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "armai_dev_silu_gate_mul_up_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "armai_dev_dequantize_q6_k": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "armai_dev_dequant_matmul_f16_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                                 c_void_p]),
    "armai_dev_int8_matmul_s32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                          c_void_p]),
    "armai_dev_int8_matmul_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_float, c_void_p,
                                          c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "armai_dev_int4_matmul_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                          c_int64, c_void_p]),
    "armai_dev_int4_gemv_q4_x_q8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                            c_int64, c_void_p]),
    "armai_dev_int4_gemv_q4_x_q8_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                            c_int64, c_void_p]),
    "armai_dev_int4_gemv_f16s": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                         c_void_p]),
    "armai_dev_rmsnorm_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                                      c_void_p]),
    "armai_dev_flash_attention_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                              c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
                                              c_void_p]),
    "armai_dev_flash_attention_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                              c_int64, c_int64, c_int64, c_int64, c_int64, c_int,
                                              c_void_p]),
    "armai_quantize_q8k": (c_int, [c_void_p, c_size_t, c_size_t, c_void_p]),
    "armai_kquant_block_dots": (c_int, [c_void_p, c_int, c_size_t, c_size_t, c_void_p, c_size_t,
                                        c_void_p, c_void_p]),
    "armai_nccl_unique_id": (c_int, [c_void_p]),
    "armai_qgemm": (c_int, [c_void_p, c_int, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p, c_float,
                            c_void_p]),
    "armai_qmatmul": (c_int, [c_void_p, c_int, c_size_t, c_size_t, c_void_p, c_size_t, c_void_p]),
    "armai_last_error": (c_char_p, []),
    "armai_version": (c_char_p, []),
}

_lock = threading.Lock()
_cuda = None
_synth = None


class ArmaiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load_cuda() -> ctypes.CDLL:
    """The CUDA library, with argument types set. Raises if it is not built."""
    global _cuda
    with _lock:
        if _cuda is None:
            if not os.path.exists(CUDA_LIB):
                raise RuntimeError(f"{CUDA_LIB} is missing: build it with `python -m arm_ai_b200.build` "
                                   "(there is no CPU fallback)")
            lib = ctypes.CDLL(CUDA_LIB)
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _cuda = lib
        return _cuda


def load_synth() -> ctypes.CDLL:
    global _synth
    with _lock:
        if _synth is None:
            if not os.path.exists(SYNTH_LIB):
                raise RuntimeError(f"{SYNTH_LIB} is missing: build it with `python -m arm_ai_b200.build`")
            lib = ctypes.CDLL(SYNTH_LIB)
            lib.synth_tensor.restype = c_int
            lib.synth_tensor.argtypes = [c_uint64, c_int64, c_int64, c_float, c_int, c_void_p]
            lib.synth_fill_normal.restype = None
            lib.synth_fill_normal.argtypes = [c_void_p, c_int64, c_uint64, c_float, c_float]
            lib.synth_quantize_q4k.restype = c_int
            lib.synth_quantize_q4k.argtypes = [c_void_p, c_int64, c_int64, c_void_p]
            lib.synth_quantize_q6k.restype = c_int
            lib.synth_quantize_q6k.argtypes = [c_void_p, c_int64, c_int64, c_void_p]
            _synth = lib
        return _synth


def last_error() -> str:
    msg = load_cuda().armai_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc != ARMAI_OK:
        raise ArmaiError(rc, last_error() or ERRORS.get(rc, f"error {rc}"))


def ptr(a) -> c_void_p:
    """Data pointer of a numpy array (or None)."""
    if a is None:
        return c_void_p(None)
    return c_void_p(a.ctypes.data)


__all__ = ["load_cuda", "load_synth", "check", "ptr", "ArmaiError", "LlamaOpts", "LlamaInfo",
           "TOKEN_CB", "c_uint16"]
