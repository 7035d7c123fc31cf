"""Mirror of the primitive NIFs (ArmAI.Native *_op, lib/arm_ai/native.ex) over
the CUDA path. Same names, argument order and return shapes as the
reference NIFs (native/arm_ai_nif/src/lib.rs:127-532, 743-764); binaries are
numpy arrays. Length mismatches raise NifError with the reference's wording.
"""
from __future__ import annotations

import numpy as np

from ._lib import load_cuda, ptr
from .native import NifError
from . import _lib


def _chk(rc):
    if rc != 0:
        raise NifError(_lib.last_error())


def _c(a, dt):
    return np.ascontiguousarray(np.asarray(a, dtype=dt).reshape(-1))


def int8_matmul_f32_op(a, w, w_scales, act_scale, m, n, k):
    a, w, ws = _c(a, np.int8), _c(w, np.int8), _c(w_scales, np.float32)
    out = np.empty(m * n, np.float32)
    _chk(load_cuda().armai_int8_matmul_f32(ptr(a), a.size, ptr(w), w.size, ptr(ws), ws.size, float(act_scale),
                                           m, n, k, ptr(out)))
    return out


def int8_matmul_f32_per_token_op(a, w, act_scales, w_scales, m, n, k):
    a, w = _c(a, np.int8), _c(w, np.int8)
    acs, ws = _c(act_scales, np.float32), _c(w_scales, np.float32)
    out = np.empty(m * n, np.float32)
    _chk(load_cuda().armai_int8_matmul_f32_per_token(ptr(a), a.size, ptr(w), w.size, ptr(acs), acs.size,
                                                     ptr(ws), ws.size, m, n, k, ptr(out)))
    return out


def int8_matmul_s32(a, w, m, n, k):
    a, w = _c(a, np.int8), _c(w, np.int8)
    out = np.empty(m * n, np.int32)
    _chk(load_cuda().armai_int8_matmul_s32(ptr(a), a.size, ptr(w), w.size, m, n, k, ptr(out)))
    return out


def quantize_int8_per_token_op(a, m, k):
    a = _c(a, np.float32)
    q = np.empty(max(m * k, 1), np.int8)
    s = np.empty(max(m, 1), np.float32)
    _chk(load_cuda().armai_quantize_int8_per_token(ptr(a), a.size, m, k, ptr(q), ptr(s)))
    return q[: m * k], s[:m]


def int4_matmul_f32_op(a, w_packed, w_scales, m, n, k):
    a, wp, ws = _c(a, np.float32), _c(w_packed, np.uint8), _c(w_scales, np.float32)
    out = np.empty(m * n, np.float32)
    _chk(load_cuda().armai_int4_matmul_f32(ptr(a), a.size, ptr(wp), wp.size, ptr(ws), ws.size, m, n, k, ptr(out)))
    return out


def int4_matmul_gemv_neon_op(a, w_packed, w_scales, n, k):
    a, wp, ws = _c(a, np.float32), _c(w_packed, np.uint8), _c(w_scales, np.float32)
    out = np.empty(n, np.float32)
    _chk(load_cuda().armai_int4_matmul_gemv(ptr(a), a.size, ptr(wp), wp.size, ptr(ws), ws.size, n, k, ptr(out)))
    return out


def int4_matmul_gemv_q4_x_q8_neon_op(a, w_packed, w_scales, n, k):
    a, wp, ws = _c(a, np.float32), _c(w_packed, np.uint8), _c(w_scales, np.float32)
    out = np.empty(n, np.float32)
    _chk(load_cuda().armai_int4_matmul_gemv_q4_x_q8(ptr(a), a.size, ptr(wp), wp.size, ptr(ws), ws.size, n, k,
                                                    ptr(out)))
    return out


def quantize_int4_q4_0_op(w, n, k):
    w = _c(w, np.float32)
    packed = np.empty(max(n * k // 2, 1), np.uint8)
    scales = np.empty(max(n * (k // 32), 1), np.float32)
    _chk(load_cuda().armai_quantize_int4_q4_0(ptr(w), w.size, n, k, ptr(packed), ptr(scales)))
    return packed[: n * k // 2], scales[: n * (k // 32)]


def rmsnorm_f32_op(input, gamma, n_outer, inner, epsilon):
    x, g = _c(input, np.float32), _c(gamma, np.float32)
    out = np.empty(max(x.size, 1), np.float32)
    _chk(load_cuda().armai_rmsnorm_f32(ptr(x), x.size, ptr(g), g.size, n_outer, inner, float(epsilon), ptr(out)))
    return out[: x.size]


def flash_attention_f32_op(q, k, v, scale, b, h, sq, sk, d, causal):
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty(max(b * h * sq * d, 1), np.float32)
    _chk(load_cuda().armai_flash_attention_f32(ptr(q), q.size, ptr(k), k.size, ptr(v), v.size, float(scale),
                                               b, h, sq, sk, d, int(bool(causal)), ptr(out)))
    return out[: b * h * sq * d]


def dequant_matmul_int8_f32_op(act, weights, scales, b, m, n, k):
    a, w, s = _c(act, np.float32), _c(weights, np.int8), _c(scales, np.float32)
    out = np.empty(max(b * m * n, 1), np.float32)
    _chk(load_cuda().armai_dequant_matmul_int8_f32(ptr(a), a.size, ptr(w), w.size, ptr(s), s.size, b, m, n, k,
                                                   ptr(out)))
    return out[: b * m * n]


# ---- LLM helper NIFs (lib.rs:147-354) ----------------------------------

def rope_f32_op(input, positions, inv_freq, n_rows, head_dim, heads_per_token):
    """rope_f32_op/6: input [n_rows, head_dim] f32, positions i64 per token,
    inv_freq [head_dim / 2] f32; interleaved pairs (shape_ops.rs:1040-1100)."""
    x, p, f = _c(input, np.float32), _c(positions, np.int64), _c(inv_freq, np.float32)
    out = np.empty(max(x.size, 1), np.float32)
    _chk(load_cuda().armai_rope_f32(ptr(x), x.size, ptr(p), p.size, ptr(f), f.size, n_rows, head_dim,
                                    heads_per_token, ptr(out)))
    return out[: x.size]


def dequant_matmul_f16_f32_op(act, weights_f16, b, m, n, k):
    """dequant_matmul_f16_f32_op/6: act [B,M,K] f32, weights [N,K] f16 (or
    their u16 bits) -> [B*M*N] f32 (shape_ops.rs:1462-1490)."""
    a = _c(act, np.float32)
    w = np.asarray(weights_f16)
    w = _c(w.view(np.uint16) if w.dtype == np.float16 else w, np.uint16)
    out = np.empty(max(b * m * n, 1), np.float32)
    _chk(load_cuda().armai_dequant_matmul_f16_f32(ptr(a), a.size, ptr(w), w.size, b, m, n, k, ptr(out)))
    return out[: b * m * n]


def softmax_last_axis_f32_op(input, outer, inner):
    """softmax_last_axis_f32_op/3 (shape_ops.rs:2719-2751)."""
    x = _c(input, np.float32)
    out = np.empty(max(x.size, 1), np.float32)
    _chk(load_cuda().armai_softmax_last_axis_f32(ptr(x), x.size, outer, inner, ptr(out)))
    return out[: x.size]


def silu_gate_mul_up_f32_op(gate, up):
    """silu_gate_mul_up_f32_op/2: silu(gate) * up (shape_ops.rs:2755-2770)."""
    g, u = _c(gate, np.float32), _c(up, np.float32)
    out = np.empty(max(g.size, 1), np.float32)
    _chk(load_cuda().armai_silu_gate_mul_up_f32(ptr(g), g.size, ptr(u), u.size, ptr(out)))
    return out[: g.size]


def dequantize_q6_k_op(input, n_elements):
    """dequantize_q6_k_op/2: GGML Q6_K bytes -> n_elements f32 (shape_ops.rs:2848-2899)."""
    b = np.frombuffer(bytes(input), np.uint8) if isinstance(input, (bytes, bytearray)) else _c(input, np.uint8)
    out = np.empty(max(n_elements, 1), np.float32)
    _chk(load_cuda().armai_dequantize_q6_k(ptr(b), b.size, n_elements, ptr(out)))
    return out[:n_elements]
