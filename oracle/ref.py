"""Python glue of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/liboracle.so`` (the C restatement in oracle.c) and feeds
it models read by gguf-py's GGUFReader — a GGUF parser independent of the one
in libarmai_cuda.so. Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import this module; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import sys
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int64, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from build import LIB, build  # noqa: E402

Q4_K, Q6_K, F32, F16 = 12, 14, 0, 1
Q4_0, Q5_0, Q8_0, Q5_K = 2, 6, 8, 13
Q8_0_DTYPE = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])
assert Q8_0_DTYPE.itemsize == 34
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = LIB if os.path.exists(LIB) else build()
        L = ctypes.CDLL(path)
        V, I64 = c_void_p, c_int64
        sigs = {
            "orc_quantize_row_q8k": (c_int, [V, I64, V]),
            "orc_vec_dot_q4k_q8k": (c_float, [I64, V, V]),
            "orc_vec_dot_q6k_q8k": (c_float, [I64, V, V]),
            "orc_dequant_row_q4k": (None, [V, I64, V]),
            "orc_dequant_row_q6k": (None, [V, I64, V]),
            "orc_q4k_block_ints": (None, [V, V, I64, V, V]),
            "orc_q6k_block_ints": (None, [V, V, I64, V]),
            "orc_qmatmul": (c_int, [V, c_int, I64, I64, V, I64, V]),
            "orc_quantize_row_q8_0": (c_int, [V, I64, V]),
            "orc_dequant_row": (c_int, [c_int, V, I64, V]),
            "orc_vec_dot_q5k_q8k": (c_float, [I64, V, V]),
            "orc_llama_new": (V, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_int]),
            "orc_llama_set_tensor": (c_int, [V, c_char_p, c_int, V, c_int, I64, I64]),
            "orc_llama_finalize": (c_int, [V]),
            "orc_llama_set_kv_f16": (None, [V, c_int]),
            "orc_llama_free": (None, [V]),
            "orc_llama_forward": (c_int, [V, V, c_int, c_int, V]),
            "orc_llama_generate": (c_int, [V, V, c_int, c_int, V, c_int, V, POINTER(c_int),
                                           POINTER(c_uint64), POINTER(c_uint64)]),
            "orc_argmax": (c_uint32, [V, I64]),
            "orc_last_error": (c_char_p, []),
            "orc_set_threads": (None, [c_int]),
            "orc_set_norm_variant": (None, [c_int]),
            "orc_get_threads": (c_int, []),
            "orc_int8_matmul_f32": (c_int, [V, V, c_float, V, I64, I64, I64, V]),
            "orc_int8_matmul_f32_per_token": (c_int, [V, V, V, V, I64, I64, I64, V]),
            "orc_int8_matmul_s32": (c_int, [V, V, I64, I64, I64, V]),
            "orc_quantize_int8_per_token": (c_int, [V, I64, I64, V, V]),
            "orc_int4_matmul_f32": (c_int, [V, V, V, I64, I64, I64, V]),
            "orc_int4_matmul_q4_x_q8": (c_int, [V, V, V, I64, I64, V]),
            "orc_quantize_int4_q4_0": (c_int, [V, I64, I64, V, V]),
            "orc_rmsnorm_f32": (c_int, [V, V, I64, I64, c_float, V]),
            "orc_flash_attention_f32": (c_int, [V, V, V, c_float, I64, I64, I64, I64, I64, c_int, V]),
            "orc_dequant_matmul_int8_f32": (c_int, [V, V, V, I64, I64, I64, I64, V]),
            "orc_rope_f32": (c_int, [V, V, V, I64, I64, I64, V]),
            "orc_softmax_last_axis_f32": (c_int, [V, I64, I64, V]),
            "orc_silu_gate_mul_up_f32": (c_int, [V, V, I64, V]),
            "orc_dequantize_q6_k": (c_int, [V, I64, V]),
            "orc_dequant_matmul_f16_f32": (c_int, [V, V, I64, I64, I64, I64, V]),
        }
        for k, (r, a) in sigs.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def P(a):
    return c_void_p(a.ctypes.data) if a is not None else c_void_p(None)


def check(rc):
    if rc != 0:
        raise RuntimeError("oracle: " + (lib().orc_last_error() or b"").decode())


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


class norm_perturbed:
    """Context manager: a last-bit perturbation of rms_norm inside the block
    (orc_set_norm_variant; variant 1 = f64 sum of squares, 2 = rms scale one
    ulp up). For measuring a model's own sensitivity, not the reference's
    arithmetic."""

    def __init__(self, variant: int = 2):
        self.variant = variant

    def __enter__(self):
        lib().orc_set_norm_variant(self.variant)
        return self

    def __exit__(self, *exc):
        lib().orc_set_norm_variant(0)
        return False


# ---------------------------------------------------------------- k-quants
def quantize_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    rows = x.reshape(-1, k)
    out = np.zeros((rows.shape[0], k // 256), dtype=Q8K_DTYPE)
    for r in range(rows.shape[0]):
        check(lib().orc_quantize_row_q8k(P(rows[r]), k, P(out[r])))
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """candle BlockQ8_0::from_float of each row (k % 32 == 0)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    rows = x.reshape(-1, k)
    out = np.zeros((rows.shape[0], k // 32), dtype=Q8_0_DTYPE)
    for r in range(rows.shape[0]):
        check(lib().orc_quantize_row_q8_0(P(rows[r]), k, P(out[r])))
    return out


def vec_dot(wtype: int, w_row: np.ndarray, q8_row: np.ndarray, k: int) -> float:
    f = {Q4_K: lib().orc_vec_dot_q4k_q8k, Q5_K: lib().orc_vec_dot_q5k_q8k}.get(wtype, lib().orc_vec_dot_q6k_q8k)
    return float(f(k, P(np.ascontiguousarray(w_row)), P(np.ascontiguousarray(q8_row))))


def dequant_rows(wtype: int, raw: np.ndarray, k: int) -> np.ndarray:
    """to_float of each row of raw GGML blocks (any type orc_dequant_row knows)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, raw.shape[-1])
    out = np.empty((raw.shape[0], k), dtype=np.float32)
    for r in range(raw.shape[0]):
        check(lib().orc_dequant_row(wtype, P(raw[r]), k, P(out[r])))
    return out


def block_ints(wtype: int, w_rows: np.ndarray, q8: np.ndarray, k: int):
    """isum[m][n][nb], msum[m][n][nb] (msum None for Q6_K)."""
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    q8 = np.ascontiguousarray(q8)
    n, nb, m = w_rows.shape[0], k // 256, q8.shape[0]
    isum = np.zeros((m, n, nb), dtype=np.int32)
    msum = np.zeros((m, n, nb), dtype=np.int32) if wtype == Q4_K else None
    for t in range(m):
        for r in range(n):
            if wtype == Q4_K:
                lib().orc_q4k_block_ints(P(w_rows[r]), P(q8[t]), nb, P(isum[t, r]), P(msum[t, r]))
            else:
                lib().orc_q6k_block_ints(P(w_rows[r]), P(q8[t]), nb, P(isum[t, r]))
    return isum, msum


def qmatmul(wtype: int, w_rows: np.ndarray, k: int, x: np.ndarray) -> np.ndarray:
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    out = np.empty((x.shape[0], w_rows.shape[0]), dtype=np.float32)
    check(lib().orc_qmatmul(P(w_rows), wtype, w_rows.shape[0], k, P(x), x.shape[0], P(out)))
    return out


# ---------------------------------------------------------------- model
class OracleLlama:
    """candle quantized_llama ModelWeights restated in C, weights from gguf-py."""

    def __init__(self, path: str, max_seq: int = 4096, kv_f16: bool = False):
        import gguf
        self.reader = gguf.GGUFReader(path)
        f = self.reader.fields

        def md(key, default=None):
            if key not in f:
                if default is not None:
                    return default
                raise KeyError(f"cannot find {key} in metadata")
            fld = f[key]
            return fld.parts[fld.data[0]][0].item()

        self.n_head = int(md("llama.attention.head_count"))
        self.n_head_kv = int(md("llama.attention.head_count_kv"))
        self.n_layer = int(md("llama.block_count"))
        self.n_embd = int(md("llama.embedding_length"))
        self.rope_dim = int(md("llama.rope.dimension_count"))
        self.eps = float(md("llama.attention.layer_norm_rms_epsilon"))
        self.rope_base = float(md("llama.rope.freq_base", 10000.0))
        self.tensors = {t.name: t for t in self.reader.tensors}
        te = self.tensors["token_embd.weight"]
        self.n_vocab = int(te.shape[1])
        self.n_ff = int(self.tensors["blk.0.ffn_gate.weight"].shape[1])
        self.max_seq = max_seq
        L = lib()
        self.h = L.orc_llama_new(self.n_layer, self.n_embd, self.n_head, self.n_head_kv, self.rope_dim,
                                 self.n_vocab, self.n_ff, self.eps, self.rope_base, max_seq)
        self._keep = []

        def put(role, layer, name):
            t = self.tensors[name]
            data = np.ascontiguousarray(t.data)
            self._keep.append(data)
            rows = int(np.prod(t.shape[1:])) if len(t.shape) > 1 else 1
            check(L.orc_llama_set_tensor(self.h, role.encode(), layer, P(data), int(t.tensor_type),
                                         rows, int(t.shape[0])))

        put("token_embd", -1, "token_embd.weight")
        put("output_norm", -1, "output_norm.weight")
        put("output", -1, "output.weight" if "output.weight" in self.tensors else "token_embd.weight")
        for l in range(self.n_layer):
            for role in ("attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                         "ffn_gate", "ffn_up", "ffn_down"):
                put(role, l, f"blk.{l}.{role}.weight")
        check(L.orc_llama_finalize(self.h))
        L.orc_llama_set_kv_f16(self.h, int(kv_f16))

    def forward(self, tokens, index_pos: int) -> np.ndarray:
        t = np.asarray(tokens, dtype=np.uint32)
        logits = np.empty(self.n_vocab, dtype=np.float32)
        check(lib().orc_llama_forward(self.h, P(t), t.size, int(index_pos), P(logits)))
        return logits

    def generate(self, prompt, max_new: int, stop_tokens=()):
        p = np.asarray(prompt, dtype=np.uint32)
        st = np.asarray(list(stop_tokens), dtype=np.uint32)
        out = np.zeros(max(max_new, 1), dtype=np.uint32)
        n = c_int(0)
        pre, dec = c_uint64(0), c_uint64(0)
        check(lib().orc_llama_generate(self.h, P(p), p.size, int(max_new), P(st) if st.size else None,
                                       st.size, P(out), ctypes.byref(n), ctypes.byref(pre),
                                       ctypes.byref(dec)))
        return [int(v) for v in out[: n.value]], int(pre.value), int(dec.value)

    def tensor_raw(self, name: str) -> np.ndarray:
        return np.ascontiguousarray(self.tensors[name].data)

    def close(self):
        if self.h:
            lib().orc_llama_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().orc_argmax(P(v), v.size))


# ---------------------------------------------------------------- primitives
def int8_matmul_f32(a, w, act_scale, w_scales, m, n, k):
    out = np.empty((m, n), dtype=np.float32)
    check(lib().orc_int8_matmul_f32(P(a), P(w), act_scale, P(w_scales), m, n, k, P(out)))
    return out


def int8_matmul_f32_per_token(a, w, act_scales, w_scales, m, n, k):
    out = np.empty((m, n), dtype=np.float32)
    check(lib().orc_int8_matmul_f32_per_token(P(a), P(w), P(act_scales), P(w_scales), m, n, k, P(out)))
    return out


def int8_matmul_s32(a, w, m, n, k):
    out = np.empty((m, n), dtype=np.int32)
    check(lib().orc_int8_matmul_s32(P(a), P(w), m, n, k, P(out)))
    return out


def quantize_int8_per_token(a, m, k):
    q = np.empty((m, k), dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    check(lib().orc_quantize_int8_per_token(P(a), m, k, P(q), P(s)))
    return q, s


def int4_matmul_f32(a, w_packed, w_scales, m, n, k):
    out = np.empty((m, n), dtype=np.float32)
    check(lib().orc_int4_matmul_f32(P(a), P(w_packed), P(w_scales), m, n, k, P(out)))
    return out


def int4_matmul_q4_x_q8(a, w_packed, w_scales, n, k):
    out = np.empty(n, dtype=np.float32)
    check(lib().orc_int4_matmul_q4_x_q8(P(a), P(w_packed), P(w_scales), n, k, P(out)))
    return out


def quantize_int4_q4_0(w, n, k):
    packed = np.empty((n, k // 2), dtype=np.uint8)
    scales = np.empty((n, k // 32), dtype=np.float32)
    check(lib().orc_quantize_int4_q4_0(P(w), n, k, P(packed), P(scales)))
    return packed, scales


def rmsnorm_f32(x, gamma, n_outer, inner, eps):
    out = np.empty((n_outer, inner), dtype=np.float32)
    check(lib().orc_rmsnorm_f32(P(x), P(gamma), n_outer, inner, eps, P(out)))
    return out


def flash_attention_f32(q, k, v, scale, b, h, sq, sk, d, causal):
    out = np.empty((b, h, sq, d), dtype=np.float32)
    check(lib().orc_flash_attention_f32(P(q), P(k), P(v), scale, b, h, sq, sk, d, int(causal), P(out)))
    return out


def dequant_matmul_int8_f32(act, w, scales, b, m, n, k):
    out = np.empty((b * m, n), dtype=np.float32)
    check(lib().orc_dequant_matmul_int8_f32(P(act), P(w), P(scales), b, m, n, k, P(out)))
    return out


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rope_f32(x, positions, inv_freq, n_rows, head_dim, heads_per_token):
    out = np.empty((n_rows, head_dim), dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    check(lib().orc_rope_f32(P(_f32(x)), P(pos), P(_f32(inv_freq)), n_rows, head_dim, heads_per_token, P(out)))
    return out


def softmax_last_axis_f32(x, outer, inner):
    out = np.empty((outer, inner), dtype=np.float32)
    check(lib().orc_softmax_last_axis_f32(P(_f32(x)), outer, inner, P(out)))
    return out


def silu_gate_mul_up_f32(gate, up):
    g, u = _f32(gate).reshape(-1), _f32(up).reshape(-1)
    out = np.empty(g.size, dtype=np.float32)
    check(lib().orc_silu_gate_mul_up_f32(P(g), P(u), g.size, P(out)))
    return out


def dequantize_q6_k(raw, n_blocks):
    b = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    out = np.empty(n_blocks * 256, dtype=np.float32)
    check(lib().orc_dequantize_q6_k(P(b), n_blocks, P(out)))
    return out


def dequant_matmul_f16_f32(act, w_bits, b, m, n, k):
    out = np.empty((b * m, n), dtype=np.float32)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    check(lib().orc_dequant_matmul_f16_f32(P(_f32(act)), P(w), b, m, n, k, P(out)))
    return out
